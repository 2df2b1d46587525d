// Internal interfaces between the C-ABI layer, the planner and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mvb {

int elem_bytes_of(int32_t dtype);

struct AttentionProblem {
  const void* query;
  int64_t q_st, q_sh;
  void* out;
  const void* cache;
  int64_t num_blocks;
  int32_t block_size, num_kv_heads, head_dim;
  const int64_t *qpos, *qstart, *qsl, *ctx_len, *table;
  int64_t table_stride, table_width;
  int64_t num_tokens, num_requests;
  int32_t num_q_heads;
  float scale;
  int32_t dtype;
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;
  cudaStream_t stream;
};

// Request classes written by the planner (one int32 per request).
enum RequestKind : int32_t {
  kKindNone = 0,     // owns no query token
  kKindDecode = 1,   // query_len * group <= kDecodeCols: split-KV decode kernel
  kKindPrefill = 2,  // longer chunks: prefill kernel
};

// Columns of the decode kernel's score tile (query tokens x heads of one
// GQA group): the N dimension of its m16n8k16 tiles.
constexpr int kDecodeCols = 8;
constexpr int kDecodeHeadDim = 128;

// Workspace carve-up.  Offsets depend only on (num_requests, num_kv_heads);
// the remaining bytes hold split-KV partials, one slot per decode item.
struct WorkspaceLayout {
  size_t ctrl, unit_prefix, kind, merge_count, partial_ml, partial_o, end_fixed;
  size_t item_bytes;
  int64_t unit_cap;  // decode units (request splits) the partial area holds
};

// ctrl[] words.
enum CtrlWord : int {
  kCtrlNumItems = 0,     // decode items = units * num_kv_heads
  kCtrlCursor = 1,       // persistent decode kernel work cursor
  kCtrlChunk = 2,        // KV tokens per split (multiple of 16)
  kCtrlNumUnits = 3,
  kCtrlPrefillCursor = 4,
  kCtrlWords = 64,
};

// Extra decode units beyond one per request that a workspace sized by
// mvb_paged_attention_workspace_size provides for splitting long contexts.
constexpr int64_t kExtraUnits = 2048;

WorkspaceLayout workspace_layout(int64_t num_requests, int32_t num_kv_heads, int32_t head_dim,
                                 size_t workspace_bytes);
size_t workspace_bytes_for(int64_t max_tokens, int64_t max_requests, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim);

int run_paged_attention(const AttentionProblem& p);

int launch_reshape_and_cache(const void* key, const int64_t* ks, const void* value,
                             const int64_t* vs, void* kv_cache, int64_t num_blocks,
                             int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                             const int64_t* slot_mapping, int64_t num_tokens, int32_t elem_bytes,
                             int32_t* status, cudaStream_t stream);

// kind_filter: NULL = every token; else only tokens of requests whose kind
// equals `want_kind` (other tokens are left untouched).
int launch_paged_attention_generic(const AttentionProblem& p, const int32_t* kind_filter,
                                   int32_t want_kind);

struct PlanTuning {
  int32_t target_items;  // aim for about this many decode items
  int32_t min_chunk;     // smallest split in KV tokens (multiple of 16)
  int32_t max_chunk;     // largest split before capacity forces more
};
PlanTuning plan_tuning();

int launch_plan(const AttentionProblem& p, const WorkspaceLayout& w, int32_t group,
                const PlanTuning& tuning);
int launch_paged_decode(const AttentionProblem& p, const WorkspaceLayout& w);

int num_sms();

}  // namespace mvb
