// Internal interfaces between the C-ABI layer, the planner and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mvb {

// cuTensorMapEncodeTiled, looked up once through the runtime's driver entry
// point (nullptr when the driver lacks it).
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled tensor_map_encoder();

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
  kKindNone = 0,     // owns no query token (or malformed)
  kKindDecode = 1,   // query_len * group <= kDecodeCols: decode kernel
  kKindPrefill = 2,  // longer chunks: prefill kernel
};

// Columns of the decode kernel's score tile (query tokens x heads of one
// GQA group): the N dimension of its m16n8k16 tiles.
constexpr int kDecodeCols = 8;
constexpr int kDecodeHeadDim = 128;
// KV heads one decode CTA streams together (a whole 2 KiB token row for
// 8 heads of 128 fp16/bf16 elements).
constexpr int kMaxHeadsPerCta = 8;
// Upper bound on decode CTAs (one or two per SM); sizes the partial area.
constexpr int kMaxDecodeCtas = 320;
// Devices the per-device host caches (SM count, grids, kernel attributes) keep.
constexpr int kMaxDevices = 64;
// Longest context a request may have (2^30 tokens).
constexpr int64_t kMaxContext = (int64_t)1 << 30;

// Status bit for a bounded wait that ran out (a kernel bug, never expected).
constexpr int32_t kStatusWaitTimeout = MVB_STATUS_WAIT_TIMEOUT;

// ctrl[] words (int64).
enum CtrlWord : int {
  kCtrlTiles = 0,          // decode tiles per KV-head group
  kCtrlPrefillUnits = 1,   // prefill query tiles (items = units x num_kv_heads)
  kCtrlPrefillCursor = 2,  // prefill work cursor (low 32 bits used)
  kCtrlWords = 32,
};

// Workspace carve-up.  Offsets depend on (num_requests, num_tokens, num_kv_heads).
struct WorkspaceLayout {
  size_t ctrl, tile_prefix, cta_start, kind, merge_count, zero_row, partial_ml, partial_o;
  size_t prefill_prefix, prefill_unit_req, prefill_unit_order, end;
};

WorkspaceLayout workspace_layout(int64_t num_requests, int64_t num_tokens, int32_t num_kv_heads);
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

// Heads a decode CTA streams: the largest divisor of num_kv_heads <= 8.
int heads_per_cta(int32_t num_kv_heads);
// Decode grid for this device and problem (also what the planner assumes).
int decode_grid(const AttentionProblem& p, int* smem_bytes);
// Arms the one-shot decode stall of mvb_debug_arm_decode_stall for this host thread.
int arm_decode_stall(int32_t cta, int32_t tile, int32_t wait_limit);

// True when the tensor-core prefill kernel can take this problem (head_dim
// 128, fp16/bf16, group dividing 128, pages of a multiple of 16 tokens,
// TMA-compatible alignment).
bool prefill_tc_supported(const AttentionProblem& p);
// Query tokens per prefill work unit (a pair of 128-row query tiles).
int prefill_tokens_per_unit(int32_t group);
int launch_paged_prefill(const AttentionProblem& p, const WorkspaceLayout& w);

struct QkPrologueArgs {
  const void* query;
  const int64_t* q_strides;
  const void* key;
  const int64_t* k_strides;
  const void* value;
  const int64_t* v_strides;
  void* q_out;
  const void* q_weight;
  const void* k_weight;
  float eps;
  const float* inv_freq;
  const int64_t* positions;
  void* kv_cache;
  int64_t num_blocks;
  int32_t block_size, num_kv_heads, head_dim;
  const int64_t* slot_mapping;
  int64_t num_tokens;
  int32_t num_q_heads, dtype;
  int32_t* status;
  cudaStream_t stream;
};
int launch_qk_prologue(const QkPrologueArgs& a);

struct SampleArgs {
  const void* logits;
  int64_t row_stride, num_rows, vocab;
  int32_t dtype;
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const uint64_t* seed;
  const int64_t* sample_index;
  int64_t* out_tokens;
  const float* noise;        // NULL: every stochastic row takes the Philox draw
  int64_t noise_stride;
  int64_t num_noise_rows;    // noise_row entries outside [0, num_noise_rows): Philox draw
  const int32_t* noise_row;
  cudaStream_t stream;
};
int launch_sample(const SampleArgs& a);

struct RmsNormArgs {
  const void* x;
  int64_t x_stride;       // elements between rows
  const void* residual;   // NULL: no residual add
  int64_t r_stride;
  void* sum_out;          // x + residual, [rows, hidden] contiguous
  void* out;              // [rows, hidden] contiguous
  const void* weight;     // [hidden]
  float eps;
  int64_t rows;
  int32_t hidden;
  int32_t dtype;
  cudaStream_t stream;
};
int launch_rms_norm(const RmsNormArgs& a);

struct SiluMulArgs {
  const void* gate_up;    // [rows, >= 2 * inter]: gate columns then up columns
  int64_t gu_stride;
  void* out;              // [rows, inter] contiguous
  int64_t rows;
  int32_t inter;
  int32_t dtype;
  cudaStream_t stream;
};
int launch_silu_mul(const SiluMulArgs& a);

struct MetadataArgs {
  const int32_t* num_computed;
  const int32_t* num_scheduled;
  const int32_t* num_block_ids;
  const int32_t* block_ids;
  const uint8_t* requires_sampling;
  const int32_t* input_token_ids;
  int64_t num_requests, num_tokens, num_block_ids_total, num_sampled;
  int64_t request_capacity, token_capacity, table_width, table_stride;
  int64_t block_size, null_block_id;
  int32_t spec_kind;
  int64_t spec_param;
  int64_t *input_ids, *positions, *context_starts, *query_start_locations, *context_lengths;
  int64_t *block_table, *slot_mapping, *sampling_rows;
  int32_t* status;
  cudaStream_t stream;
};
constexpr int64_t kMaxMetadataRequests = 16384;  // shared-memory offsets of every request
int launch_build_metadata(const MetadataArgs& a);

int launch_plan(const AttentionProblem& p, const WorkspaceLayout& w, int32_t group,
                int32_t decode_ctas, int32_t prefill_block_q);
int launch_paged_decode(const AttentionProblem& p, const WorkspaceLayout& w, int32_t grid,
                        int32_t smem_bytes);

int num_sms();

}  // namespace mvb
