// Exact CUDA-core paged attention for every shape the tensor-core kernels do
// not take: any head_dim up to 256, any block size, any GQA ratio, and fp32.
//
// One warp owns one (query token, query head) row.  It finds the token's
// request by binary search over query_start_locations (the same ownership
// rule as _find_request_for_query_block, triton_paged.py:71-94, applied per
// token), then walks the visible keys in position order, reading each key
// through the block table (reference.py:101-138 gathers the same positions)
// and keeping an fp32 online softmax (max, sum, weighted V).  Lanes split the
// head dimension; the q.k dot product is a warp shuffle reduction.
//
// Visible keys of token t in request r (reference.py:49-68):
//   lo = max(ctx_start[qsl[r]], ctx_start[t], 0)
//   hi = min(context_lengths[r] - 1, pos[t])
// Softmax is computed as exp2((s - max) * log2e) with the scale folded in;
// a request whose gathered history is empty gives 0 (einsum over an empty
// axis), a token with an empty window gives NaN (softmax of all -inf).
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kMaxDimPerLane = 8;  // head_dim <= 256

template <typename T>
__global__ void __launch_bounds__(128) paged_attention_generic_kernel(
    const T* __restrict__ query, int64_t q_st, int64_t q_sh, T* __restrict__ out,
    const T* __restrict__ cache, int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
    int32_t head_dim, const int64_t* __restrict__ qpos, const int64_t* __restrict__ qstart,
    const int64_t* __restrict__ qsl, const int64_t* __restrict__ ctx_len,
    const int64_t* __restrict__ table, int64_t table_stride, int64_t table_width,
    int64_t num_tokens, int64_t num_requests, int32_t num_q_heads, float scale_log2,
    const int32_t* __restrict__ kind_filter, int32_t want_kind, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= num_tokens * num_q_heads) return;
  const int64_t t = row / num_q_heads;
  const int32_t hq = (int32_t)(row % num_q_heads);
  const int32_t group = num_q_heads / num_kv_heads;
  const int32_t h = hq / group;
  T* orow = out + row * head_dim;

  const int64_t r = find_request(qsl, num_requests, t);
  if (kind_filter != nullptr && (r < 0 || __ldg(kind_filter + r) != want_kind)) return;
  if (r < 0) {
    for (int d = lane; d < head_dim; d += 32) orow[d] = from_float<T>(0.f);
    return;
  }
  const int64_t first = __ldg(qsl + r);
  const int64_t gather_lo = __ldg(qstart + first);
  const int64_t clen = __ldg(ctx_len + r);
  if (clen - gather_lo <= 0) {  // empty gathered history
    for (int d = lane; d < head_dim; d += 32) orow[d] = from_float<T>(0.f);
    return;
  }
  int64_t lo = max(gather_lo, __ldg(qstart + t));
  lo = max(lo, (int64_t)0);
  const int64_t hi = min(clen - 1, __ldg(qpos + t));

  float q[kMaxDimPerLane], acc[kMaxDimPerLane];
  const T* qrow = query + t * q_st + (int64_t)hq * q_sh;
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) {
    const int d = lane + 32 * i;
    q[i] = d < head_dim ? to_float(qrow[d]) : 0.f;
    acc[i] = 0.f;
  }
  const int64_t plane = num_blocks * block_size * num_kv_heads * head_dim;
  const int64_t* trow = table + r * table_stride;
  float m = -INFINITY, l = 0.f;
  for (int64_t p = lo; p <= hi; ++p) {
    const int64_t lb = p / block_size;
    const int64_t blk = lb < table_width ? __ldg(trow + lb) : -1;
    if (blk < 0 || blk >= num_blocks) {
      if (status != nullptr && lane == 0) atomicOr(status, MVB_STATUS_BLOCK_OUT_OF_RANGE);
      continue;
    }
    const int64_t base = ((blk * block_size + p % block_size) * num_kv_heads + h) * head_dim;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < head_dim) dot += q[i] * to_float(cache[base + d]);
    }
    const float s = warp_sum(dot) * scale_log2;
    const float m_new = fmaxf(m, s);
    const float corr = exp2f(m - m_new);  // m = -inf on the first key: corr = 0
    const float pw = exp2f(s - m_new);
    l = l * corr + pw;
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) {
      const int d = lane + 32 * i;
      const float v = d < head_dim ? to_float(cache[plane + base + d]) : 0.f;
      acc[i] = acc[i] * corr + pw * v;
    }
    m = m_new;
  }
  // l == 0 (no visible key) yields 0/0 = NaN, matching softmax over all -inf.
  const float inv = 1.f / l;
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < head_dim) orow[d] = from_float<T>(l > 0.f ? acc[i] * inv : NAN);
  }
}

}  // namespace

int launch_paged_attention_generic(const AttentionProblem& p, const int32_t* kind_filter,
                                   int32_t want_kind) {
  if (p.num_tokens == 0) return MVB_OK;
  if (p.head_dim > 32 * kMaxDimPerLane) return MVB_ERR_UNSUPPORTED_SHAPE;
  const int64_t rows = p.num_tokens * p.num_q_heads;
  const int64_t blocks = (rows + 3) / 4;
  if (blocks > 0x7fffffffLL) return MVB_ERR_UNSUPPORTED_SHAPE;
  const float scale_log2 = p.scale * 1.4426950408889634f;
#define MVB_GENERIC_LAUNCH(T)                                                                 \
  paged_attention_generic_kernel<T><<<(unsigned)blocks, 128, 0, p.stream>>>(                  \
      static_cast<const T*>(p.query), p.q_st, p.q_sh, static_cast<T*>(p.out),                 \
      static_cast<const T*>(p.cache), p.num_blocks, p.block_size, p.num_kv_heads, p.head_dim, \
      p.qpos, p.qstart, p.qsl, p.ctx_len, p.table, p.table_stride, p.table_width,             \
      p.num_tokens, p.num_requests, p.num_q_heads, scale_log2, kind_filter, want_kind, p.status)
  switch (p.dtype) {
    case MVB_DTYPE_F16:
      MVB_GENERIC_LAUNCH(__half);
      break;
    case MVB_DTYPE_BF16:
      MVB_GENERIC_LAUNCH(__nv_bfloat16);
      break;
    case MVB_DTYPE_F32:
      MVB_GENERIC_LAUNCH(float);
      break;
    default:
      return MVB_ERR_UNSUPPORTED_DTYPE;
  }
#undef MVB_GENERIC_LAUNCH
  return check_launch();
}

}  // namespace mvb
