// Device-side build of one step's attention metadata from per-request counts.
//
// The reference model runner builds a step's batch on the host
// (worker/model_runner.py:751-900): a Python loop over the scheduled requests
// for positions, query start locations, context lengths and sampling rows;
// per request a torch.arange and a block-id tensor for the slot mapping
// (map_cache_slots, attention/attention.py:31-41); per request a row copy
// into a null-padded block table; then a per-position host loop for each
// cache group's visibility starts (Attention.build_metadata,
// attention/attention.py:56-85, spec.py).  When a CUDA graph replays the step,
// _CudaGraphExecution.copy_input (model_runner.py:78-122) pads everything to
// the captured capacity.  Here the host uploads four int32 arrays (counts,
// concatenated block ids, optionally token ids and sampling flags) and one
// launch writes every int64 output, padded to the capacity exactly as
// copy_input pads it:
//   input_ids / positions / context starts: 0 past num_tokens,
//   query_start_locations: num_tokens past num_requests + 1,
//   context_lengths: 0 past num_requests,
//   block_table: null_block_id past each request's block ids and rows,
//   slot_mapping: -1 past num_tokens.
//
// Every CTA scans the per-request counts into shared-memory offsets (the
// counts are a few KB and stay in L2), then the grid writes tokens, table
// rows and request entries with grid-stride loops: no inter-CTA dependency.
#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kMetaThreads = 512;
constexpr int kMetaWarps = kMetaThreads / 32;

// Inclusive warp scan of three int64 sums.
__device__ __forceinline__ void warp_scan3(int64_t& a, int64_t& b, int64_t& c, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t ua = __shfl_up_sync(0xffffffffu, a, o);
    const int64_t ub = __shfl_up_sync(0xffffffffu, b, o);
    const int64_t uc = __shfl_up_sync(0xffffffffu, c, o);
    if (lane >= o) {
      a += ua;
      b += ub;
      c += uc;
    }
  }
}

__device__ __forceinline__ int64_t context_start_of(int64_t pos, int32_t kind, int64_t param) {
  if (kind == MVB_SPEC_SLIDING_WINDOW) {  // SlidingWindowSpec.context_start (spec.py)
    const int64_t s = pos - param + 1;
    return s > 0 ? s : 0;
  }
  if (kind == MVB_SPEC_CHUNKED_LOCAL) return (pos / param) * param;  // ChunkedLocalSpec
  return 0;                                                         // FullAttentionSpec
}

__global__ void __launch_bounds__(kMetaThreads)
    build_metadata_kernel(const MetadataArgs a) {
  extern __shared__ int32_t meta_smem[];
  const int64_t R = a.num_requests;
  int32_t* off_tok = meta_smem;            // [R + 1] first token of each request
  int32_t* off_blk = off_tok + (R + 1);    // [R + 1] first block id of each request
  int32_t* off_smp = off_blk + (R + 1);    // [R + 1] first sampling row of each request
  __shared__ int64_t warp_tot[3][kMetaWarps];
  __shared__ int64_t totals[3];
  __shared__ int bad_sh;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) bad_sh = 0;
  __syncthreads();

  // 1. Counts into shared memory (coalesced), checked.
  int bad = 0;
  for (int64_t i = tid; i < R; i += kMetaThreads) {
    const int32_t n = a.num_scheduled[i], b = a.num_block_ids[i], c = a.num_computed[i];
    bad |= (n < 0) | (b < 0) | (c < 0) | ((int64_t)b > a.table_width);
    off_tok[i] = n;
    off_blk[i] = b;
    off_smp[i] = a.requires_sampling ? (a.requires_sampling[i] != 0) : 0;
  }
  if (bad) bad_sh = 1;
  __syncthreads();

  // 2. Exclusive scan: each thread owns a contiguous segment.
  const int64_t per = (R + kMetaThreads - 1) / kMetaThreads;
  const int64_t lo = tid * per, hi = lo + per < R ? lo + per : R;
  int64_t sa = 0, sb = 0, sc = 0;
  for (int64_t i = lo; i < hi; ++i) {
    sa += off_tok[i];
    sb += off_blk[i];
    sc += off_smp[i];
  }
  int64_t ia = sa, ib = sb, ic = sc;
  warp_scan3(ia, ib, ic, lane);
  if (lane == 31) {
    warp_tot[0][warp] = ia;
    warp_tot[1][warp] = ib;
    warp_tot[2][warp] = ic;
  }
  __syncthreads();
  if (warp == 0) {
    int64_t wa = lane < kMetaWarps ? warp_tot[0][lane] : 0;
    int64_t wb = lane < kMetaWarps ? warp_tot[1][lane] : 0;
    int64_t wc = lane < kMetaWarps ? warp_tot[2][lane] : 0;
    warp_scan3(wa, wb, wc, lane);
    if (lane < kMetaWarps) {  // exclusive prefix of the warps before
      warp_tot[0][lane] = wa - warp_tot[0][lane];
      warp_tot[1][lane] = wb - warp_tot[1][lane];
      warp_tot[2][lane] = wc - warp_tot[2][lane];
    }
    if (lane == 31) {
      totals[0] = wa;
      totals[1] = wb;
      totals[2] = wc;
    }
  }
  __syncthreads();
  int64_t ra = warp_tot[0][warp] + ia - sa, rb = warp_tot[1][warp] + ib - sb,
          rc = warp_tot[2][warp] + ic - sc;
  for (int64_t i = lo; i < hi; ++i) {
    const int32_t na = off_tok[i], nb = off_blk[i], nc = off_smp[i];
    off_tok[i] = (int32_t)ra;
    off_blk[i] = (int32_t)rb;
    off_smp[i] = (int32_t)rc;
    ra += na;
    rb += nb;
    rc += nc;
  }
  if (tid == 0) {
    off_tok[R] = (int32_t)totals[0];
    off_blk[R] = (int32_t)totals[1];
    off_smp[R] = (int32_t)totals[2];
  }
  __syncthreads();
  // The sizes the host passed must be the sums of the counts; only then are
  // the 32-bit offsets exact (the host sizes are below 2^31).
  const bool valid = !bad_sh && totals[0] == a.num_tokens && totals[1] == a.num_block_ids_total &&
                     totals[2] == a.num_sampled;
  if (!valid && blockIdx.x == 0 && tid == 0 && a.status)
    atomicOr(a.status, MVB_STATUS_INCONSISTENT_COUNTS);

  const int64_t T = valid ? a.num_tokens : 0;  // real tokens; the rest is padding
  const int64_t Rv = valid ? R : 0;            // real requests
  const int64_t gthreads = (int64_t)gridDim.x * kMetaThreads;
  const int64_t gtid = (int64_t)blockIdx.x * kMetaThreads + tid;

  // 3. Tokens: position, token id, visibility start, cache slot.
  int past = 0;
  for (int64_t t = gtid; t < a.token_capacity; t += gthreads) {
    int64_t pos = 0, start = 0, slot = -1, id = 0;
    if (t < T) {
      int32_t l = 0, h = (int32_t)R;  // largest r with off_tok[r] <= t
      while (h - l > 1) {
        const int32_t m = (l + h) >> 1;
        if (off_tok[m] <= t)
          l = m;
        else
          h = m;
      }
      const int32_t r = l;
      pos = (int64_t)a.num_computed[r] + (t - off_tok[r]);
      start = context_start_of(pos, a.spec_kind, a.spec_param);
      const int64_t logical = pos / a.block_size;
      if (logical < off_blk[r + 1] - off_blk[r])
        slot = (int64_t)a.block_ids[off_blk[r] + logical] * a.block_size + pos % a.block_size;
      else
        past = 1;  // map_cache_slots would raise IndexError
      if (a.input_token_ids) id = a.input_token_ids[t];
    }
    if (a.positions) a.positions[t] = pos;
    if (a.context_starts) a.context_starts[t] = start;
    if (a.slot_mapping) a.slot_mapping[t] = slot;
    if (a.input_ids) a.input_ids[t] = id;
  }
  if (__any_sync(0xffffffffu, past) && lane == 0 && a.status)
    atomicOr(a.status, MVB_STATUS_POSITION_PAST_TABLE);

  // 4. Block-table rows, one warp per row (coalesced), null-padded.
  if (a.block_table) {
    const int64_t gwarp = (int64_t)blockIdx.x * kMetaWarps + warp;
    const int64_t nwarps = (int64_t)gridDim.x * kMetaWarps;
    for (int64_t r = gwarp; r < a.request_capacity; r += nwarps) {
      int64_t* row = a.block_table + r * a.table_stride;
      const int64_t first = r < Rv ? off_blk[r] : 0;
      const int64_t n = r < Rv ? off_blk[r + 1] - off_blk[r] : 0;
      for (int64_t j = lane; j < a.table_width; j += 32)
        row[j] = j < n ? (int64_t)a.block_ids[first + j] : a.null_block_id;
    }
  }

  // 5. Per-request entries and the sampled rows.
  for (int64_t r = gtid; r <= a.request_capacity; r += gthreads) {
    if (a.query_start_locations) a.query_start_locations[r] = r <= Rv ? off_tok[r] : a.num_tokens;
    if (r == a.request_capacity) break;
    if (a.context_lengths)
      a.context_lengths[r] = r < Rv ? (int64_t)a.num_computed[r] + (off_tok[r + 1] - off_tok[r]) : 0;
    if (r < Rv && a.sampling_rows && off_smp[r + 1] > off_smp[r])
      a.sampling_rows[off_smp[r]] = (int64_t)off_tok[r + 1] - 1;
  }
}

}  // namespace

int launch_build_metadata(const MetadataArgs& a) {
  const size_t smem = (size_t)3 * (size_t)(a.num_requests + 1) * sizeof(int32_t);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(build_metadata_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return MVB_ERR_CUDA;
    }
  }
  const int64_t table_cells = a.block_table ? a.request_capacity * a.table_width : 0;
  int64_t want = (a.token_capacity + 1023) / 1024;
  want = want > (table_cells + 4095) / 4096 ? want : (table_cells + 4095) / 4096;
  want = want > (a.request_capacity + 1 + 1023) / 1024 ? want : (a.request_capacity + 1 + 1023) / 1024;
  const int64_t cap = 2 * (int64_t)num_sms();
  const int grid = (int)(want < 1 ? 1 : (want > cap ? cap : want));
  build_metadata_kernel<<<grid, kMetaThreads, smem, a.stream>>>(a);
  return check_launch();
}

}  // namespace mvb
