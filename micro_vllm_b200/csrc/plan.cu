// Device-side batch planner: turns the metadata tensors into the decode
// kernel's work decomposition without a host round trip, so a step can be
// captured in a CUDA graph and replayed with new metadata.
//
// Block 0 classifies every request and lays the KV of all decode-class
// requests out as one sequence of 16-token tiles (per request: the
// positions from its visibility start rounded down to 16, to its context
// length).  It writes the per-request tile prefix sums and, for each decode
// CTA b, the request holding the first tile of b's equal share
// [b*N/G, (b+1)*N/G) of the N tiles — the stream-K split the decode kernel
// walks.  The other blocks zero the output rows of tokens owned by no
// request (graph padding), which the Triton backend gets from
// torch.zeros_like (triton_paged.py:343).
#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kPlanThreads = 1024;

struct PlanParams {
  const int64_t* qsl;
  const int64_t* qstart;
  const int64_t* qpos;
  const int64_t* ctx_len;
  int64_t num_requests;
  int64_t num_tokens;
  int32_t group;
  int32_t num_q_heads;
  int32_t head_dim;
  int32_t elem_bytes;
  int32_t num_kv_heads;
  int32_t heads_per_cta;
  int32_t decode_ctas;
  int32_t prefill_block_q;  // 0: prefill-class requests go to the CUDA-core kernel
  void* out;
  int64_t* ctrl;
  int64_t* tile_prefix;
  int32_t* cta_start;
  int32_t* kind;
  int32_t* merge_count;
  uint4* zero_row;
  int64_t* prefill_prefix;
  int32_t* prefill_unit_req;
  int32_t* prefill_unit_order;
};

// Units are ordered by their number of visible keys in 128-key tiles
// (counting sort, largest first); longer ones share a bucket.
constexpr int kOrderBuckets = 2048;

// Class and decode tile count of request r.
__device__ __forceinline__ int64_t request_tiles(const PlanParams& p, int64_t r, int32_t* kind) {
  const int64_t qs = p.qsl[r], qe = p.qsl[r + 1];
  const int64_t len = qe - qs;
  // Zero-length (graph padding) or malformed ranges own no work.
  if (len <= 0 || qs < 0 || qe > p.num_tokens) {
    *kind = kKindNone;
    return 0;
  }
  const int64_t hi = p.ctx_len[r];
  if (hi > kMaxContext) {  // beyond any pool: refuse rather than overflow
    *kind = kKindNone;
    return 0;
  }
  if (len * p.group > kDecodeCols) {
    *kind = kKindPrefill;
    return 0;
  }
  const int64_t lo = max(p.qstart[qs], (int64_t)0);
  *kind = kKindDecode;
  const int64_t span = hi > lo ? hi - (lo & ~(int64_t)15) : 0;
  return span > 0 ? (span + 15) >> 4 : 1;  // an empty history still owns one (empty) tile
}

// Block-wide inclusive scan of one int64 per thread (1024 threads).
__device__ __forceinline__ int64_t block_inclusive_scan(int64_t v, int64_t* warp_tot,
                                                        int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int64_t w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_tot[lane] = w;  // inclusive warp prefix
    if (lane == 31) *total = w;
  }
  __syncthreads();
  const int64_t res = v + (warp > 0 ? warp_tot[warp - 1] : 0);
  __syncthreads();
  return res;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanParams p) {
  // The decode kernel is launched as a programmatic dependent: it may set up
  // on the free SMs now and waits for this grid before reading the plan.
  allow_dependent_launch();
  if (blockIdx.x > 0) {
    // Zero rows of tokens outside [qsl[0], qsl[R]).
    const int64_t covered_lo =
        p.num_requests > 0 ? min(max(p.qsl[0], (int64_t)0), p.num_tokens) : 0;
    const int64_t covered_hi =
        p.num_requests > 0 ? min(max(p.qsl[p.num_requests], covered_lo), p.num_tokens) : 0;
    const int64_t row_words = (int64_t)p.num_q_heads * p.head_dim * p.elem_bytes / 4;
    const int64_t head = covered_lo * row_words;
    const int64_t tail = (p.num_tokens - covered_hi) * row_words;
    uint32_t* out = static_cast<uint32_t*>(p.out);
    for (int64_t i = (int64_t)(blockIdx.x - 1) * blockDim.x + threadIdx.x; i < head + tail;
         i += (int64_t)(gridDim.x - 1) * blockDim.x) {
      out[i < head ? i : covered_hi * row_words + (i - head)] = 0u;
    }
    return;
  }

  __shared__ int64_t warp_tot[32];
  __shared__ int64_t total;
  __shared__ int32_t bucket[kOrderBuckets];
  // A copy of tile_prefix for the decode CTAs' searches below (batches of up
  // to kSmemPrefix requests), so they read shared rather than global memory.
  constexpr int kSmemPrefix = 2048;
  __shared__ int64_t prefix_sh[kSmemPrefix + 1];
  const bool prefix_in_smem = p.num_requests <= kSmemPrefix;

  // Per-request decode tile counts and prefill query-tile counts, and their
  // exclusive prefix sums.
  int64_t running = 0, running_units = 0;
  for (int64_t base = 0; base < p.num_requests; base += kPlanThreads) {
    const int64_t r = base + threadIdx.x;
    int64_t tiles = 0, units = 0;
    if (r < p.num_requests) {
      int32_t k;
      tiles = request_tiles(p, r, &k);
      p.kind[r] = k;
      if (k == kKindPrefill && p.prefill_block_q > 0)
        units = (p.qsl[r + 1] - p.qsl[r] + p.prefill_block_q - 1) / p.prefill_block_q;
    }
    const int64_t incl = block_inclusive_scan(tiles, warp_tot, &total);
    if (r < p.num_requests) {
      p.tile_prefix[r] = running + incl - tiles;
      if (prefix_in_smem) prefix_sh[r] = running + incl - tiles;
    }
    running += total;
    __syncthreads();
    const int64_t incl_u = block_inclusive_scan(units, warp_tot, &total);
    const int64_t first_unit = running_units + incl_u - units;
    if (r < p.num_requests) {
      p.prefill_prefix[r] = first_unit;
      for (int64_t u = 0; u < units; ++u) p.prefill_unit_req[first_unit + u] = (int32_t)r;
    }
    running_units += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    p.tile_prefix[p.num_requests] = running;
    if (prefix_in_smem) prefix_sh[p.num_requests] = running;
    p.prefill_prefix[p.num_requests] = running_units;
    p.ctrl[kCtrlTiles] = running;
    p.ctrl[kCtrlPrefillUnits] = running_units;
    p.ctrl[kCtrlPrefillCursor] = 0;
  }
  for (int64_t i = threadIdx.x; i < p.num_requests * p.num_kv_heads; i += kPlanThreads)
    p.merge_count[i] = 0;

  // Prefill units, longest first, so the prefill kernel's work cursor hands
  // out the long query tiles before the short ones and the CTAs finish
  // together.  Work of a unit ~ the keys its last token sees.
  if (running_units > 0) {
    for (int i = threadIdx.x; i < kOrderBuckets; i += kPlanThreads) bucket[i] = 0;
    __syncthreads();
    auto unit_bucket = [&](int64_t u) -> int32_t {
      const int64_t r = p.prefill_unit_req[u];
      const int64_t qs = p.qsl[r], qe = p.qsl[r + 1];
      const int64_t first = qs + (u - p.prefill_prefix[r]) * p.prefill_block_q;
      const int64_t last = min(first + p.prefill_block_q, qe) - 1;
      const int64_t lo = max(max(p.qstart[qs], (int64_t)0), min(p.qstart[first], p.qstart[last]));
      const int64_t hi = min(p.ctx_len[r] - 1, p.qpos[last]);
      const int64_t tiles = hi >= lo ? ((hi - lo) >> 7) + 1 : 0;
      return (int32_t)(kOrderBuckets - 1 - min(tiles, (int64_t)kOrderBuckets - 1));  // descending
    };
    for (int64_t u = threadIdx.x; u < running_units; u += kPlanThreads)
      atomicAdd(&bucket[unit_bucket(u)], 1);
    __syncthreads();
    // Exclusive scan of the bucket counts (2 per thread).
    {
      const int i0 = 2 * threadIdx.x;
      const int64_t c0 = bucket[i0], c1 = bucket[i0 + 1];
      const int64_t incl = block_inclusive_scan(c0 + c1, warp_tot, &total);
      __syncthreads();
      bucket[i0] = (int32_t)(incl - c0 - c1);
      bucket[i0 + 1] = (int32_t)(incl - c1);
    }
    __syncthreads();
    for (int64_t u = threadIdx.x; u < running_units; u += kPlanThreads)
      p.prefill_unit_order[atomicAdd(&bucket[unit_bucket(u)], 1)] = (int32_t)u;
  }
  if (threadIdx.x < kMaxHeadsPerCta * 256 / 16) p.zero_row[threadIdx.x] = make_uint4(0, 0, 0, 0);
  __syncthreads();  // tile_prefix complete before the searches below

  // Request holding the first tile of each decode CTA's share.
  const int64_t groups = p.num_kv_heads / p.heads_per_cta;
  const int64_t n_all = running * groups;
  for (int b = threadIdx.x; b < p.decode_ctas; b += kPlanThreads) {
    const int64_t first = (int64_t)b * n_all / p.decode_ctas;
    int32_t r_first = 0;
    if (running > 0 && first < n_all) {
      const int64_t local = first % running;
      int64_t lo = 0, hi = p.num_requests;  // largest r with tile_prefix[r] <= local
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((prefix_in_smem ? prefix_sh[mid] : p.tile_prefix[mid]) <= local)
          lo = mid + 1;
        else
          hi = mid;
      }
      r_first = (int32_t)(lo - 1);
    }
    p.cta_start[b] = r_first;
  }
}

}  // namespace

int launch_plan(const AttentionProblem& a, const WorkspaceLayout& w, int32_t group,
                int32_t decode_ctas, int32_t prefill_block_q) {
  char* ws = static_cast<char*>(a.workspace);
  PlanParams p;
  p.qsl = a.qsl;
  p.qstart = a.qstart;
  p.qpos = a.qpos;
  p.ctx_len = a.ctx_len;
  p.num_requests = a.num_requests;
  p.num_tokens = a.num_tokens;
  p.group = group;
  p.num_q_heads = a.num_q_heads;
  p.head_dim = a.head_dim;
  p.elem_bytes = elem_bytes_of(a.dtype);
  p.num_kv_heads = a.num_kv_heads;
  p.heads_per_cta = heads_per_cta(a.num_kv_heads);
  p.decode_ctas = decode_ctas;
  p.prefill_block_q = prefill_block_q;
  p.out = a.out;
  p.ctrl = reinterpret_cast<int64_t*>(ws + w.ctrl);
  p.tile_prefix = reinterpret_cast<int64_t*>(ws + w.tile_prefix);
  p.cta_start = reinterpret_cast<int32_t*>(ws + w.cta_start);
  p.kind = reinterpret_cast<int32_t*>(ws + w.kind);
  p.merge_count = reinterpret_cast<int32_t*>(ws + w.merge_count);
  p.zero_row = reinterpret_cast<uint4*>(ws + w.zero_row);
  p.prefill_prefix = reinterpret_cast<int64_t*>(ws + w.prefill_prefix);
  p.prefill_unit_req = reinterpret_cast<int32_t*>(ws + w.prefill_unit_req);
  p.prefill_unit_order = reinterpret_cast<int32_t*>(ws + w.prefill_unit_order);
  // Block 0 plans; 32 more blocks zero padding rows (enough for a few MB).
  plan_kernel<<<33, kPlanThreads, 0, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
