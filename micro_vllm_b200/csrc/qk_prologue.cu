// Fused attention prologue of a Qwen3 layer: per-head RMSNorm of the query
// and key heads, rotary position embedding of both, and the KV-cache write
// (rotated key, raw value) — one launch instead of norm, norm, rotary and
// write.  Restates, step for step in the same dtypes:
//   Qwen3Attention.forward q/k norm then rope  (models/qwen.py:74-98)
//   RMSNorm.forward                             (layers/normalization.py:15-22)
//   rotate_half / RotaryEmbedding.forward       (layers/rotary_embedding.py:7-11, 22-52)
//   write_kv_cache                              (attention/operators/reference.py:84-98)
// fp32 statistics; the normalised value is rounded to the model dtype before
// the weight multiply (computed in fp32 — exact for two 16-bit operands —
// and rounded again); the rotation is fp32 with separately rounded products
// and sum (no fused multiply-add, as the reference's elementwise ops); the
// result is rounded to the model dtype.  Rotary inverse frequencies come in
// precomputed (the caller evaluates the reference's own expression), so the
// angles are the reference's bit for bit.
//
// One warp per token: it evaluates the token's rotation angles once, then
// walks its rows — the Hq query heads, the Hkv key heads, the Hkv value
// heads — in batches of 8 loaded together.  A lane owns 4 consecutive
// elements of the 128-element row, so rotate_half's partner of lane l is
// lane l ^ 16.
// Roofline: HBM; bytes per token = (Hq + 2 Hkv) * D * elsize read +
// (Hq + 2 Hkv) * D * elsize written.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kRowsPerWarp = 8;
constexpr int kPrologueWarps = 8;
constexpr int kPrologueDim = 128;

struct PrologueParams {
  const char* q;
  int64_t q_st, q_sh;  // element strides (token, head); unit dim stride
  const char* k;
  int64_t k_st, k_sh;
  const char* v;
  int64_t v_st, v_sh;
  char* q_out;  // [T, Hq, 128] contiguous
  const char* q_w;
  const char* k_w;
  float eps;
  const float* inv_freq;  // [64]
  const int64_t* pos;
  char* cache;  // [2, num_slots, Hkv, 128]
  int64_t num_slots;
  const int64_t* slots;
  int64_t num_tokens;
  int32_t num_q_heads, num_kv_heads;
  int32_t* status;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
// Round through the model dtype.
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return to_f<T>(from_f<T>(v));
}

// 4 consecutive 16-bit elements as one 8-byte word.
template <typename T>
__device__ __forceinline__ void unpack4(uint2 w, float (&x)[4]) {
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = to_f<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ uint2 pack4(const float (&x)[4]) {
  uint2 w;
  T* e = reinterpret_cast<T*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) e[i] = from_f<T>(x[i]);
  return w;
}

template <typename T>
__global__ void __launch_bounds__(32 * kPrologueWarps)
    qk_prologue_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kPrologueWarps + (threadIdx.x >> 5);
  if (t >= p.num_tokens) return;
  const int rows = p.num_q_heads + 2 * p.num_kv_heads;
  const int qk_rows = p.num_q_heads + p.num_kv_heads;

  const int64_t slot = __ldg(p.slots + t);
  const bool write = slot >= 0 && slot < p.num_slots;
  if (slot >= p.num_slots && lane == 0 && p.status != nullptr)
    atomicOr(p.status, MVB_STATUS_SLOT_OUT_OF_RANGE);

  // Rotation of this lane's columns 4*lane..4*lane+3, once per token:
  // column c and c + 64 share frequency c mod 64 (angles = cat(freqs, freqs)).
  float cs[4], sn[4], qw[4], kw[4];
  {
    const float pf = (float)__ldg(p.pos + t);  // positions.to(float32)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float ang = __fmul_rn(pf, __ldg(p.inv_freq + ((4 * lane + i) & 63)));
      sincosf(ang, &sn[i], &cs[i]);
    }
    unpack4<T>(__ldg(reinterpret_cast<const uint2*>(p.q_w) + lane), qw);
    unpack4<T>(__ldg(reinterpret_cast<const uint2*>(p.k_w) + lane), kw);
  }

  for (int r0 = 0; r0 < rows; r0 += kRowsPerWarp) {
    const int nr = min(kRowsPerWarp, rows - r0);
    // A batch of rows in flight at once.
    uint2 raw[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      raw[i] = make_uint2(0, 0);
      if (i < nr) {
        const int r = r0 + i;
        const char* base;
        if (r < p.num_q_heads)
          base = p.q + (t * p.q_st + (int64_t)r * p.q_sh) * 2;
        else if (r < qk_rows)
          base = p.k + (t * p.k_st + (int64_t)(r - p.num_q_heads) * p.k_sh) * 2;
        else
          base = p.v + (t * p.v_st + (int64_t)(r - qk_rows) * p.v_sh) * 2;
        raw[i] = __ldg(reinterpret_cast<const uint2*>(base) + lane);
      }
    }
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      if (i >= nr) break;
      const int r = r0 + i;
      if (r >= qk_rows) {  // value row: straight into plane 1
        if (write) {
          char* dst = p.cache + ((p.num_slots + slot) * p.num_kv_heads + (r - qk_rows)) *
                                    (int64_t)kPrologueDim * 2;
          reinterpret_cast<uint2*>(dst)[lane] = raw[i];
        }
        continue;
      }
      const bool is_q = r < p.num_q_heads;
      float x[4];
      unpack4<T>(raw[i], x);
      // RMSNorm: mean of squares over the row, fp32.
      float ss = x[0] * x[0];
      ss = __fadd_rn(ss, __fmul_rn(x[1], x[1]));
      ss = __fadd_rn(ss, __fmul_rn(x[2], x[2]));
      ss = __fadd_rn(ss, __fmul_rn(x[3], x[3]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      const float inv_rms = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / kPrologueDim), p.eps));
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        y[e] = rnd<T>(__fmul_rn(is_q ? qw[e] : kw[e], rnd<T>(__fmul_rn(x[e], inv_rms))));
      // rotate_half: the first half takes -x[c + 64], the second x[c - 64].
      float out[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, y[e], 16);
        const float rot = lane < 16 ? -partner : partner;
        out[e] = __fadd_rn(__fmul_rn(y[e], cs[e]), __fmul_rn(rot, sn[e]));
      }
      const uint2 w = pack4<T>(out);
      if (is_q) {
        reinterpret_cast<uint2*>(p.q_out + ((t * p.num_q_heads + r) * (int64_t)kPrologueDim) * 2)[lane] = w;
      } else if (write) {
        char* dst = p.cache + (slot * p.num_kv_heads + (r - p.num_q_heads)) * (int64_t)kPrologueDim * 2;
        reinterpret_cast<uint2*>(dst)[lane] = w;
      }
    }
  }
}

}  // namespace

int launch_qk_prologue(const QkPrologueArgs& a) {
  if (a.head_dim != kPrologueDim) return MVB_ERR_UNSUPPORTED_SHAPE;
  auto aligned8 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 7) == 0; };
  // Rows move as 8-byte words: every row start must be 8-byte aligned.
  const bool strides_ok = a.q_strides[2] == 1 && a.k_strides[2] == 1 && a.v_strides[2] == 1 &&
                          a.q_strides[0] % 4 == 0 && a.q_strides[1] % 4 == 0 &&
                          a.k_strides[0] % 4 == 0 && a.k_strides[1] % 4 == 0 &&
                          a.v_strides[0] % 4 == 0 && a.v_strides[1] % 4 == 0;
  if (!strides_ok || !aligned8(a.query) || !aligned8(a.key) || !aligned8(a.value) ||
      !aligned8(a.q_out) || !aligned8(a.q_weight) || !aligned8(a.k_weight) || !aligned8(a.kv_cache))
    return MVB_ERR_UNSUPPORTED_SHAPE;
  PrologueParams p;
  p.q = static_cast<const char*>(a.query);
  p.q_st = a.q_strides[0];
  p.q_sh = a.q_strides[1];
  p.k = static_cast<const char*>(a.key);
  p.k_st = a.k_strides[0];
  p.k_sh = a.k_strides[1];
  p.v = static_cast<const char*>(a.value);
  p.v_st = a.v_strides[0];
  p.v_sh = a.v_strides[1];
  p.q_out = static_cast<char*>(a.q_out);
  p.q_w = static_cast<const char*>(a.q_weight);
  p.k_w = static_cast<const char*>(a.k_weight);
  p.eps = a.eps;
  p.inv_freq = a.inv_freq;
  p.pos = a.positions;
  p.cache = static_cast<char*>(a.kv_cache);
  p.num_slots = a.num_blocks * a.block_size;
  p.slots = a.slot_mapping;
  p.num_tokens = a.num_tokens;
  p.num_q_heads = a.num_q_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.status = a.status;
  const int64_t blocks = (a.num_tokens + kPrologueWarps - 1) / kPrologueWarps;
  if (blocks > INT32_MAX) return MVB_ERR_UNSUPPORTED_SHAPE;
  if (a.dtype == MVB_DTYPE_BF16)
    qk_prologue_kernel<__nv_bfloat16><<<(unsigned)blocks, 32 * kPrologueWarps, 0, a.stream>>>(p);
  else
    qk_prologue_kernel<__half><<<(unsigned)blocks, 32 * kPrologueWarps, 0, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
