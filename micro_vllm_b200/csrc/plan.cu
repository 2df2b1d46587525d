// Device-side batch planner: turns the metadata tensors into the decode
// kernel's work decomposition without a host round trip, so a step can be
// captured in a CUDA graph and replayed with new metadata.
//
// Block 0 classifies every request, picks the split size and writes, per
// request, the prefix sum of its decode units (KV splits).  Decode item i
// is unit i / num_kv_heads of KV head i % num_kv_heads, so consecutive items
// are the KV heads of the same pages: CTAs that run together read adjacent
// 256-byte head rows of one 2 KiB token row.  The remaining blocks zero the
// output rows of tokens that belong to no request (graph padding), which the
// Triton backend gets from torch.zeros_like (triton_paged.py:343).
#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kPlanThreads = 1024;
// Longest context a request may have (2^30 tokens); keeps split sizes in int32.
constexpr int64_t kMaxContext = (int64_t)1 << 30;

struct PlanParams {
  const int64_t* qsl;
  const int64_t* qstart;
  const int64_t* ctx_len;
  int64_t num_requests;
  int64_t num_tokens;
  int32_t num_kv_heads;
  int32_t group;
  int32_t num_q_heads;
  int32_t head_dim;
  int32_t elem_bytes;
  void* out;
  int32_t* ctrl;
  int32_t* unit_prefix;
  int32_t* kind;
  int32_t* merge_count;
  int64_t unit_cap;
  PlanTuning tuning;
};

// Aligned KV extent of decode-class request r: [base, hi) with base = lo
// rounded down to 16 so that 16-token tiles line up with 16-token pages.
__device__ __forceinline__ void request_extent(const PlanParams& p, int64_t r, int32_t* kind,
                                               int64_t* span) {
  const int64_t qs = p.qsl[r], qe = p.qsl[r + 1];
  const int64_t len = qe - qs;
  *span = 0;
  // Zero-length (graph padding) or malformed ranges own no work.
  if (len <= 0 || qs < 0 || qe > p.num_tokens) {
    *kind = kKindNone;
    return;
  }
  if (len * p.group > kDecodeCols) {
    *kind = kKindPrefill;
    return;
  }
  *kind = kKindDecode;
  const int64_t lo = max(p.qstart[qs], (int64_t)0);
  const int64_t hi = p.ctx_len[r];
  if (hi > kMaxContext) {  // beyond any pool: refuse rather than overflow
    *kind = kKindNone;
    return;
  }
  *span = hi > lo ? hi - (lo & ~(int64_t)15) : 0;
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
  if (blockIdx.x > 0) {
    // Zero rows of tokens outside [qsl[0], qsl[R]).
    const int64_t covered_lo = p.num_requests > 0 ? min(max(p.qsl[0], (int64_t)0), p.num_tokens) : 0;
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
  __shared__ int64_t red[2];

  // Pass 1: total aligned decode span and number of decode requests.
  int64_t span_sum = 0, dec_count = 0;
  for (int64_t r = threadIdx.x; r < p.num_requests; r += kPlanThreads) {
    int32_t k;
    int64_t span;
    request_extent(p, r, &k, &span);
    p.kind[r] = k;
    span_sum += span;
    dec_count += (k == kKindDecode);
  }
  if (threadIdx.x < 2) red[threadIdx.x] = 0;
  __syncthreads();
  atomicAdd(reinterpret_cast<unsigned long long*>(&red[0]), (unsigned long long)span_sum);
  atomicAdd(reinterpret_cast<unsigned long long*>(&red[1]), (unsigned long long)dec_count);
  __syncthreads();
  span_sum = red[0];
  dec_count = red[1];

  // Split size: about target_items items over all KV heads, clamped, then
  // raised until sum(ceil(span/chunk)) <= span_sum/chunk + dec_count fits.
  int64_t chunk = (span_sum * p.num_kv_heads + p.tuning.target_items - 1) / p.tuning.target_items;
  chunk = max(chunk, (int64_t)p.tuning.min_chunk);
  chunk = min(chunk, (int64_t)p.tuning.max_chunk);
  const int64_t room = p.unit_cap - dec_count;  // >= 1, checked by the host
  chunk = max(chunk, (span_sum + room - 1) / max(room, (int64_t)1));
  chunk = max((chunk + 15) & ~(int64_t)15, (int64_t)16);

  // Pass 2: per-request unit counts and their exclusive prefix sum.
  int64_t running = 0;
  for (int64_t base = 0; base < p.num_requests; base += kPlanThreads) {
    const int64_t r = base + threadIdx.x;
    int64_t units = 0;
    if (r < p.num_requests) {
      int32_t k;
      int64_t span;
      request_extent(p, r, &k, &span);
      if (k == kKindDecode) units = span > 0 ? (span + chunk - 1) / chunk : 1;
    }
    const int64_t incl = block_inclusive_scan(units, warp_tot, &total);
    if (r < p.num_requests) p.unit_prefix[r] = (int32_t)(running + incl - units);
    running += total;
    __syncthreads();
  }
  for (int64_t i = threadIdx.x; i < p.num_requests * p.num_kv_heads; i += kPlanThreads)
    p.merge_count[i] = 0;
  if (threadIdx.x == 0) {
    p.unit_prefix[p.num_requests] = (int32_t)running;
    p.ctrl[kCtrlNumUnits] = (int32_t)running;
    p.ctrl[kCtrlNumItems] = (int32_t)(running * p.num_kv_heads);
    p.ctrl[kCtrlCursor] = 0;
    p.ctrl[kCtrlPrefillCursor] = 0;
    p.ctrl[kCtrlChunk] = (int32_t)chunk;
  }
}

}  // namespace

int launch_plan(const AttentionProblem& a, const WorkspaceLayout& w, int32_t group,
                const PlanTuning& tuning) {
  char* ws = static_cast<char*>(a.workspace);
  PlanParams p;
  p.qsl = a.qsl;
  p.qstart = a.qstart;
  p.ctx_len = a.ctx_len;
  p.num_requests = a.num_requests;
  p.num_tokens = a.num_tokens;
  p.num_kv_heads = a.num_kv_heads;
  p.group = group;
  p.num_q_heads = a.num_q_heads;
  p.head_dim = a.head_dim;
  p.elem_bytes = elem_bytes_of(a.dtype);
  p.out = a.out;
  p.ctrl = reinterpret_cast<int32_t*>(ws + w.ctrl);
  p.unit_prefix = reinterpret_cast<int32_t*>(ws + w.unit_prefix);
  p.kind = reinterpret_cast<int32_t*>(ws + w.kind);
  p.merge_count = reinterpret_cast<int32_t*>(ws + w.merge_count);
  p.unit_cap = w.unit_cap;
  p.tuning = tuning;
  // Block 0 plans; 32 more blocks zero padding rows (enough for a few MB).
  plan_kernel<<<33, kPlanThreads, 0, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
