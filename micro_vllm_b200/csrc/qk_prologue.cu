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
// One warp per token.  It copies the token's Hkv value rows to the cache (16
// bytes per lane, two rows per instruction), evaluates its rotation angles
// once, then walks its Hq query rows and its Hkv key rows in batches of 8
// loaded together.  A lane owns columns 2l, 2l+1 and 2l+64, 2l+65 of the
// 128-element row, so rotate_half's partner of every column is in the same
// lane; the 8 rows of a batch share one transposed warp reduction of their
// statistics.  The fp32 arithmetic runs on packed pairs (mul/sub/add/fma
// .rn.f32x2: each half rounded as the scalar op), which halves the
// instructions of the norm and the rotation; the kernel is issue-bound
// without them.
// Roofline: HBM; bytes per token = (Hq + 2 Hkv) * D * elsize read +
// (Hq + 2 Hkv) * D * elsize written.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"
#include "ptx_sm100.cuh"

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

// Two adjacent 16-bit elements as one 32-bit word, and the paired ops on them.
template <typename T>
struct Pair;
template <>
struct Pair<__half> {
  static __device__ __forceinline__ float2 to_f2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  // Correctly rounded product of two 16-bit values (exact in fp32, one rounding).
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const __half2 h = __hmul2_rn(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <>
struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_f2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const __nv_bfloat162 h = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                        *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

// Sum over the warp of 8 per-lane values s[0..7], transposed: lane l ends
// with the total of value (l >> 2) & 7.  9 shuffles for 8 rows instead of 40.
__device__ __forceinline__ float reduce8_transposed(const float (&s)[8], int lane) {
  float t[4], u[2];
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = b16 ? s[i + 4] : s[i], send = b16 ? s[i] : s[i + 4];
    t[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b8 ? t[i + 2] : t[i], send = b8 ? t[i] : t[i + 2];
    u[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float v = (b4 ? u[1] : u[0]) + __shfl_xor_sync(0xffffffffu, b4 ? u[0] : u[1], 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  sm100::f32x2_unpack(v, r.x, r.y);
  return r;
}

// n rows (head stride `sh` bytes from `src`) normalised with weight words
// (w_lo, w_hi), rotated, and stored to consecutive 256-byte rows at `dst`.
template <typename T>
__device__ __forceinline__ void norm_rope_rows(const char* src, int64_t sh, int n, char* dst, bool store,
                                               uint32_t w_lo, uint32_t w_hi, uint64_t cs, uint64_t sn,
                                               float eps, int lane) {
  using P = Pair<T>;
  for (int r0 = 0; r0 < n; r0 += kRowsPerWarp) {
    const int nr = min(kRowsPerWarp, n - r0);
    uint32_t lo[kRowsPerWarp], hi[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      lo[i] = hi[i] = 0;
      if (i < nr) {
        const uint32_t* row = reinterpret_cast<const uint32_t*>(src + (int64_t)(r0 + i) * sh);
        lo[i] = __ldg(row + lane);
        hi[i] = __ldg(row + 32 + lane);
      }
    }
    // RMSNorm statistics of the batch's rows: per-lane sums of squares
    // (fp32), then one transposed warp reduction and one reciprocal root per
    // lane for all 8 rows; row i's factor is then read from lane 4i.
    float ss[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const float2 a = P::to_f2(lo[i]), b = P::to_f2(hi[i]);
      const uint64_t av = sm100::f32x2_pack(a.x, a.y), bv = sm100::f32x2_pack(b.x, b.y);
      const float2 s2 = unpack2(sm100::f32x2_fma(bv, bv, sm100::f32x2_mul(av, av)));
      ss[i] = s2.x + s2.y;
    }
    const float tot = reduce8_transposed(ss, lane);
    const float inv_lane = 1.0f / sqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / kPrologueDim), eps));
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const float inv_rms = __shfl_sync(0xffffffffu, inv_lane, 4 * i);
      if (i >= nr) break;
      const uint64_t inv2 = sm100::f32x2_pack(inv_rms, inv_rms);
      const float2 a = P::to_f2(lo[i]), b = P::to_f2(hi[i]);
      // The normalised value rounded to the model dtype, times the weight
      // (one correctly rounded 16-bit product).
      const float2 na = unpack2(sm100::f32x2_mul(sm100::f32x2_pack(a.x, a.y), inv2));
      const float2 nb = unpack2(sm100::f32x2_mul(sm100::f32x2_pack(b.x, b.y), inv2));
      const float2 ya = P::to_f2(P::mul(P::from_f2(na.x, na.y), w_lo));
      const float2 yb = P::to_f2(P::mul(P::from_f2(nb.x, nb.y), w_hi));
      const uint64_t yav = sm100::f32x2_pack(ya.x, ya.y), ybv = sm100::f32x2_pack(yb.x, yb.y);
      // x * cos + rotate_half(x) * sin, products and sums rounded separately.
      const float2 o_lo = unpack2(sm100::f32x2_sub(sm100::f32x2_mul(yav, cs), sm100::f32x2_mul(ybv, sn)));
      const float2 o_hi = unpack2(sm100::f32x2_add(sm100::f32x2_mul(ybv, cs), sm100::f32x2_mul(yav, sn)));
      if (store) {
        uint32_t* d = reinterpret_cast<uint32_t*>(dst + (int64_t)(r0 + i) * (kPrologueDim * 2));
        d[lane] = P::from_f2(o_lo.x, o_lo.y);
        d[32 + lane] = P::from_f2(o_hi.x, o_hi.y);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(32 * kPrologueWarps)
    qk_prologue_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kPrologueWarps + (threadIdx.x >> 5);
  if (t >= p.num_tokens) return;

  const int64_t slot = __ldg(p.slots + t);
  const bool write = slot >= 0 && slot < p.num_slots;
  if (slot >= p.num_slots && lane == 0 && p.status != nullptr)
    atomicOr(p.status, MVB_STATUS_SLOT_OUT_OF_RANGE);

  constexpr int64_t kRowBytes = kPrologueDim * 2;
  const char* vbase = p.v + t * p.v_st * 2;
  char* kcache = p.cache + (write ? slot : 0) * p.num_kv_heads * kRowBytes;
  char* vcache = p.cache + (p.num_slots + (write ? slot : 0)) * p.num_kv_heads * kRowBytes;

  // Value rows go to plane 1 unchanged: 16 bytes per lane, two rows per
  // instruction when the rows are 16-byte aligned, else 8 bytes per lane.
  if (write) {
    const int64_t vsh = p.v_sh * 2;
    if (((reinterpret_cast<uintptr_t>(vbase) | (uintptr_t)vsh | reinterpret_cast<uintptr_t>(vcache)) & 15) == 0) {
      const int half = lane >> 4, col = lane & 15;
      for (int h0 = 0; h0 < p.num_kv_heads; h0 += 8) {
        uint4 w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int h = h0 + 2 * i + half;
          if (h < p.num_kv_heads) w[i] = __ldg(reinterpret_cast<const uint4*>(vbase + h * vsh) + col);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int h = h0 + 2 * i + half;
          if (h < p.num_kv_heads) reinterpret_cast<uint4*>(vcache + h * kRowBytes)[col] = w[i];
        }
      }
    } else {
      for (int h = 0; h < p.num_kv_heads; ++h)
        reinterpret_cast<uint2*>(vcache + h * kRowBytes)[lane] =
            __ldg(reinterpret_cast<const uint2*>(vbase + h * vsh) + lane);
    }
  }

  // Lane l owns columns 2l, 2l+1 (word l of the row) and 2l+64, 2l+65 (word
  // l+32): rotate_half pairs column c with c + 64, so both partners sit in
  // one lane, and c and c + 64 share frequency c (angles = cat(freqs, freqs)).
  float cs[2], sn[2];
  {
    const float pf = (float)__ldg(p.pos + t);  // positions.to(float32)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float ang = __fmul_rn(pf, __ldg(p.inv_freq + 2 * lane + i));
      sincosf(ang, &sn[i], &cs[i]);
    }
  }
  const uint64_t csv = sm100::f32x2_pack(cs[0], cs[1]), snv = sm100::f32x2_pack(sn[0], sn[1]);
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(p.q_w);
  const uint32_t* kw = reinterpret_cast<const uint32_t*>(p.k_w);
  norm_rope_rows<T>(p.q + t * p.q_st * 2, p.q_sh * 2, p.num_q_heads, p.q_out + t * p.num_q_heads * kRowBytes,
                    true, __ldg(qw + lane), __ldg(qw + 32 + lane), csv, snv, p.eps, lane);
  norm_rope_rows<T>(p.k + t * p.k_st * 2, p.k_sh * 2, p.num_kv_heads, kcache, write, __ldg(kw + lane),
                    __ldg(kw + 32 + lane), csv, snv, p.eps, lane);
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
