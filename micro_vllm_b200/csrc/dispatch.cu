// run_paged_attention: picks the kernels for one call and carves the
// caller's workspace.  Nothing here touches device memory from the host.
#include <stdlib.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {

namespace {

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  if (v == nullptr || *v == '\0') return fallback;
  const int x = atoi(v);
  return x > 0 ? x : fallback;
}

}  // namespace

WorkspaceLayout workspace_layout(int64_t num_requests, int32_t num_kv_heads, int32_t head_dim,
                                 size_t workspace_bytes) {
  WorkspaceLayout w;
  size_t off = 0;
  w.ctrl = off;
  off += align256(kCtrlWords * sizeof(int32_t));
  w.unit_prefix = off;
  off += align256((size_t)(num_requests + 1) * sizeof(int32_t));
  w.kind = off;
  off += align256((size_t)num_requests * sizeof(int32_t));
  w.merge_count = off;
  off += align256((size_t)num_requests * num_kv_heads * sizeof(int32_t));
  w.end_fixed = off;
  w.item_bytes = (size_t)kDecodeCols * ((size_t)head_dim * sizeof(float) + sizeof(float2));
  const size_t room = workspace_bytes > off + 256 ? workspace_bytes - off - 256 : 0;
  w.unit_cap = (int64_t)(room / (w.item_bytes * num_kv_heads));
  w.partial_ml = off;
  w.partial_o =
      off + align256((size_t)w.unit_cap * num_kv_heads * kDecodeCols * sizeof(float2));
  return w;
}

size_t workspace_bytes_for(int64_t max_tokens, int64_t max_requests, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim) {
  (void)max_tokens;
  (void)num_q_heads;
  const WorkspaceLayout w = workspace_layout(max_requests, num_kv_heads, head_dim, 0);
  return w.end_fixed + 512 + (size_t)(max_requests + kExtraUnits) * num_kv_heads * w.item_bytes;
}

PlanTuning plan_tuning() {
  static const PlanTuning t = {
      env_int("MVB_DECODE_TARGET_ITEMS", 4096),
      (env_int("MVB_DECODE_MIN_CHUNK", 64) + 15) & ~15,
      (env_int("MVB_DECODE_MAX_CHUNK", 1024) + 15) & ~15,
  };
  return t;
}

int num_sms() {
  static int cached_device = -1, cached = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached = n;
    cached_device = dev;
  }
  return cached;
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
  const WorkspaceLayout w =
      workspace_layout(p.num_requests, p.num_kv_heads, p.head_dim, p.workspace_bytes);
  if (w.unit_cap < p.num_requests + 1) return MVB_ERR_WORKSPACE_TOO_SMALL;

  int rc = launch_plan(p, w, group, plan_tuning());
  if (rc != MVB_OK) return rc;
  rc = launch_paged_decode(p, w);
  if (rc != MVB_OK) return rc;
  // Requests whose query chunk does not fit the decode tile.
  const int32_t* kind = reinterpret_cast<const int32_t*>(static_cast<char*>(p.workspace) + w.kind);
  return launch_paged_attention_generic(p, kind, kKindPrefill);
}

}  // namespace mvb
