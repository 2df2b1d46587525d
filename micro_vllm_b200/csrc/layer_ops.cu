// Element-wise stages of a Qwen3 decoder layer that the reference model runs
// as chains of small torch kernels, one launch each here:
//   RMSNorm.forward                     (layers/normalization.py:15-22): the
//     row in fp32, its mean square, times 1/sqrt(mean + eps), rounded to the
//     model dtype, times the weight (the 16-bit product is exact in fp32, so
//     one rounding);
//   the residual add before it          (models/qwen.py:151-154): the sum of
//     two 16-bit values in fp32, rounded to the model dtype, as torch's add;
//   SwiGLUMLP's silu(gate) * up         (layers/mlp.py:19-21): silu in fp32
//     (x / (1 + exp(-x))), rounded, times up (exact in fp32), rounded.
// The sums of squares are added in another order than torch's reduction (as
// any parallel sum); everything else rounds where the reference rounds.
// Roofline: HBM; both kernels read and write each element once (RMSNorm reads
// its row twice, the second time from L1).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kNormWarps = 8;   // rows per CTA
constexpr int kVec = 8;         // 16-bit elements per 16-byte access

template <typename T>
struct Elem;
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float2 to_f2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_f2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

// x + residual, rounded to T, for the 8 elements of one 16-byte word pair.
template <typename T>
__device__ __forceinline__ uint4 add8(uint4 x, uint4 r) {
  using E = Elem<T>;
  uint4 o;
  const uint32_t* xa = reinterpret_cast<const uint32_t*>(&x);
  const uint32_t* ra = reinterpret_cast<const uint32_t*>(&r);
  uint32_t* oa = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = E::to_f2(xa[i]), b = E::to_f2(ra[i]);
    oa[i] = E::from_f2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
  }
  return o;
}

struct NormParams {
  const char* x;
  int64_t x_stride;  // elements between rows
  const char* residual;  // NULL: plain RMSNorm
  int64_t r_stride;
  char* sum_out;  // x + residual (with residual)
  char* out;      // [T, H] contiguous
  const char* weight;
  float eps;
  int64_t rows;
  int32_t hidden;
};

// One warp per row: pass 1 the sum of squares (and the residual sum, stored),
// pass 2 the normalised, weighted row (the row's words again, from L1).
template <typename T, bool kAdd>
__global__ void __launch_bounds__(32 * kNormWarps) rms_norm_kernel(const NormParams p) {
  using E = Elem<T>;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nvec = p.hidden / kVec;
  const uint4* x = reinterpret_cast<const uint4*>(p.x + row * p.x_stride * 2);
  const uint4* r = kAdd ? reinterpret_cast<const uint4*>(p.residual + row * p.r_stride * 2) : nullptr;
  uint4* sum_out = kAdd ? reinterpret_cast<uint4*>(p.sum_out + row * (int64_t)p.hidden * 2) : nullptr;
  float ss = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    uint4 h = __ldg(x + v);
    if constexpr (kAdd) {
      h = add8<T>(h, __ldg(r + v));
      sum_out[v] = h;
    }
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = E::to_f2(hw[i]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  // mean = sum x (1 / H), as torch's mean; then 1 / sqrt(mean + eps).
  const float inv = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)p.hidden), p.eps));
  const uint4* w = reinterpret_cast<const uint4*>(p.weight);
  uint4* out = reinterpret_cast<uint4*>(p.out + row * (int64_t)p.hidden * 2);
  for (int v = lane; v < nvec; v += 32) {
    uint4 h = __ldg(x + v);
    if constexpr (kAdd) h = add8<T>(h, __ldg(r + v));
    const uint4 wv = __ldg(w + v);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = E::to_f2(hw[i]);
      // Normalised value rounded to T, then the weight product (exact in
      // fp32 for two 16-bit operands) rounded once.
      const float2 y = E::to_f2(E::from_f2(__fmul_rn(f.x, inv), __fmul_rn(f.y, inv)));
      const float2 g = E::to_f2(ww[i]);
      ow[i] = E::from_f2(__fmul_rn(g.x, y.x), __fmul_rn(g.y, y.y));
    }
    out[v] = o;
  }
}

struct SiluMulParams {
  const char* gate_up;  // [T, 2I]: gate columns, then up columns
  int64_t gu_stride;    // elements between rows
  char* out;            // [T, I] contiguous
  int64_t rows;
  int32_t inter;
};

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluMulParams p) {
  using E = Elem<T>;
  const int64_t per_row = p.inter / kVec;
  const int64_t total = p.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row, v = i - row * per_row;
    const uint4* src = reinterpret_cast<const uint4*>(p.gate_up + row * p.gu_stride * 2);
    const uint4 g = __ldg(src + v), u = __ldg(src + per_row + v);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = E::to_f2(gw[k]), b = E::to_f2(uw[k]);
      // silu in fp32, rounded to T; then the product with up, rounded once.
      const float2 s = E::to_f2(E::from_f2(__fdiv_rn(a.x, __fadd_rn(1.0f, expf(-a.x))),
                                           __fdiv_rn(a.y, __fadd_rn(1.0f, expf(-a.y)))));
      ow[k] = E::from_f2(__fmul_rn(s.x, b.x), __fmul_rn(s.y, b.y));
    }
    reinterpret_cast<uint4*>(p.out + row * (int64_t)p.inter * 2)[v] = o;
  }
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace

int launch_rms_norm(const RmsNormArgs& a) {
  if (a.hidden <= 0 || a.hidden % kVec != 0 || a.rows < 0) return MVB_ERR_UNSUPPORTED_SHAPE;
  if (a.rows == 0) return MVB_OK;
  const bool add = a.residual != nullptr;
  if (!aligned16(a.x) || !aligned16(a.out) || !aligned16(a.weight) || a.x_stride % kVec != 0 ||
      (add && (!aligned16(a.residual) || !aligned16(a.sum_out) || a.r_stride % kVec != 0)))
    return MVB_ERR_UNSUPPORTED_SHAPE;
  NormParams p;
  p.x = static_cast<const char*>(a.x);
  p.x_stride = a.x_stride;
  p.residual = static_cast<const char*>(a.residual);
  p.r_stride = a.r_stride;
  p.sum_out = static_cast<char*>(a.sum_out);
  p.out = static_cast<char*>(a.out);
  p.weight = static_cast<const char*>(a.weight);
  p.eps = a.eps;
  p.rows = a.rows;
  p.hidden = a.hidden;
  const int64_t blocks = (a.rows + kNormWarps - 1) / kNormWarps;
  if (blocks > INT32_MAX) return MVB_ERR_UNSUPPORTED_SHAPE;
  const dim3 grid((unsigned)blocks), block(32 * kNormWarps);
  if (a.dtype == MVB_DTYPE_BF16) {
    if (add)
      rms_norm_kernel<__nv_bfloat16, true><<<grid, block, 0, a.stream>>>(p);
    else
      rms_norm_kernel<__nv_bfloat16, false><<<grid, block, 0, a.stream>>>(p);
  } else {
    if (add)
      rms_norm_kernel<__half, true><<<grid, block, 0, a.stream>>>(p);
    else
      rms_norm_kernel<__half, false><<<grid, block, 0, a.stream>>>(p);
  }
  return check_launch();
}

int launch_silu_mul(const SiluMulArgs& a) {
  if (a.inter <= 0 || a.inter % kVec != 0 || a.rows < 0) return MVB_ERR_UNSUPPORTED_SHAPE;
  if (a.rows == 0) return MVB_OK;
  if (!aligned16(a.gate_up) || !aligned16(a.out) || a.gu_stride % kVec != 0 || a.gu_stride < 2 * (int64_t)a.inter)
    return MVB_ERR_UNSUPPORTED_SHAPE;
  SiluMulParams p;
  p.gate_up = static_cast<const char*>(a.gate_up);
  p.gu_stride = a.gu_stride;
  p.out = static_cast<char*>(a.out);
  p.rows = a.rows;
  p.inter = a.inter;
  const int64_t work = a.rows * (a.inter / kVec);
  const int64_t cap = (int64_t)num_sms() * 8;  // 8 CTAs of 256 threads per SM, grid-stride beyond
  const int64_t blocks = (work + 255) / 256 < cap ? (work + 255) / 256 : cap;
  if (a.dtype == MVB_DTYPE_BF16)
    silu_mul_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, a.stream>>>(p);
  else
    silu_mul_kernel<__half><<<(unsigned)blocks, 256, 0, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
