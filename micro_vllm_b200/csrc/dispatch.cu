// run_paged_attention: picks the kernels for one call and carves the
// caller's workspace.  Nothing here touches device memory from the host.
#include <mutex>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {

namespace {

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

WorkspaceLayout workspace_layout(int64_t num_requests, int64_t num_tokens, int32_t num_kv_heads) {
  WorkspaceLayout w;
  size_t off = 0;
  w.ctrl = off;
  off += align256(kCtrlWords * sizeof(int64_t));
  w.tile_prefix = off;
  off += align256((size_t)(num_requests + 1) * sizeof(int64_t));
  w.cta_start = off;
  off += align256((size_t)kMaxDecodeCtas * sizeof(int32_t));
  w.kind = off;
  off += align256((size_t)num_requests * sizeof(int32_t));
  w.merge_count = off;
  off += align256((size_t)num_requests * num_kv_heads * sizeof(int32_t));
  w.zero_row = off;
  off += align256((size_t)kMaxHeadsPerCta * kDecodeHeadDim * 2);
  const size_t partials = (size_t)kMaxDecodeCtas * 2 * kMaxHeadsPerCta * kDecodeCols;
  w.partial_ml = off;
  off += align256(partials * sizeof(float2));
  w.partial_o = off;
  off += align256(partials * kDecodeHeadDim * sizeof(float));
  w.prefill_prefix = off;
  off += align256((size_t)(num_requests + 1) * sizeof(int64_t));
  w.prefill_unit_req = off;  // at most one prefill unit per token plus one per request
  off += align256((size_t)(num_tokens + num_requests) * sizeof(int32_t));
  w.prefill_unit_order = off;  // the same units, most keys first
  off += align256((size_t)(num_tokens + num_requests) * sizeof(int32_t));
  w.end = off;
  return w;
}

size_t workspace_bytes_for(int64_t max_tokens, int64_t max_requests, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim) {
  (void)num_q_heads;
  (void)head_dim;
  return workspace_layout(max_requests, max_tokens, num_kv_heads).end;
}

int num_sms() {
  // One entry per device, filled under a lock: host threads driving
  // different devices may call at the same time.
  static std::mutex lock;
  static int cached[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool slot = dev >= 0 && dev < kMaxDevices;
  std::lock_guard<std::mutex> guard(lock);
  if (!slot || cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    if (!slot) return n;
    cached[dev] = n;
  }
  return cached[dev];
}

int run_paged_attention(const AttentionProblem& p) {
  const int32_t group = p.num_q_heads / p.num_kv_heads;
  const bool half_type = p.dtype == MVB_DTYPE_F16 || p.dtype == MVB_DTYPE_BF16;
  const bool aligned = ((uintptr_t)p.query % 4) == 0 && (p.q_st % 2) == 0 &&
                       (p.q_sh % 2) == 0 && ((uintptr_t)p.out % 4) == 0 &&
                       ((uintptr_t)p.cache % 16) == 0;
  const bool fast = half_type && p.head_dim == kDecodeHeadDim && aligned;
  if (!fast) return launch_paged_attention_generic(p, nullptr, 0);

  if (p.workspace == nullptr || ((uintptr_t)p.workspace % 256) != 0)
    return MVB_ERR_INVALID_ARGUMENT;
  const WorkspaceLayout w = workspace_layout(p.num_requests, p.num_tokens, p.num_kv_heads);
  if (p.workspace_bytes < w.end) return MVB_ERR_WORKSPACE_TOO_SMALL;
  int smem = 0;
  const int grid = decode_grid(p, &smem);
  if (grid <= 0) return MVB_ERR_CUDA;

  const bool tc_prefill = prefill_tc_supported(p);
  int rc = launch_plan(p, w, group, grid, tc_prefill ? prefill_tokens_per_unit(group) : 0);
  if (rc != MVB_OK) return rc;
  rc = launch_paged_decode(p, w, grid, smem);
  if (rc != MVB_OK) return rc;
  // Requests whose query chunk does not fit the decode tile.
  if (tc_prefill) return launch_paged_prefill(p, w);
  const int32_t* kind = reinterpret_cast<const int32_t*>(static_cast<char*>(p.workspace) + w.kind);
  return launch_paged_attention_generic(p, kind, kKindPrefill);
}

}  // namespace mvb
