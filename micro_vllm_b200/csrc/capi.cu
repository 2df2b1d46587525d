// extern "C" entry points declared in include/mvb200.h: argument checks,
// dtype/shape dispatch and error reporting.  No entry point allocates,
// synchronises or reads device memory from the host.
#include <stdio.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {

namespace {
thread_local int g_last_cuda_error = 0;
}

void set_last_cuda_error(cudaError_t err) { g_last_cuda_error = (int)err; }

int check_launch() {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return MVB_ERR_CUDA;
  }
  return MVB_OK;
}

int elem_bytes_of(int32_t dtype) {
  switch (dtype) {
    case MVB_DTYPE_F16:
    case MVB_DTYPE_BF16:
      return 2;
    case MVB_DTYPE_F32:
      return 4;
    default:
      return 0;
  }
}

}  // namespace mvb

using namespace mvb;

extern "C" {

int mvb_version(void) { return (0 << 16) | 1; }

const char* mvb_status_string(int status) {
  switch (status) {
    case MVB_OK:
      return "ok";
    case MVB_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case MVB_ERR_UNSUPPORTED_DTYPE:
      return "unsupported dtype";
    case MVB_ERR_UNSUPPORTED_SHAPE:
      return "unsupported shape";
    case MVB_ERR_WORKSPACE_TOO_SMALL:
      return "workspace too small";
    case MVB_ERR_CUDA:
      return "CUDA error";
    default:
      return "unknown status";
  }
}

int mvb_last_cuda_error(void) { return g_last_cuda_error; }

int mvb_debug_arm_decode_stall(int32_t cta, int32_t tile, int32_t wait_limit) {
  return arm_decode_stall(cta, tile, wait_limit);
}

int mvb_reshape_and_cache(const void* key, const int64_t* key_strides, const void* value,
                          const int64_t* value_strides, void* kv_cache, int64_t num_blocks,
                          int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                          const int64_t* slot_mapping, int64_t num_tokens, int32_t dtype,
                          int32_t* status, void* stream) {
  const int eb = elem_bytes_of(dtype);
  if (eb == 0) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens < 0 || num_blocks < 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MVB_OK;
  if (!key || !value || !kv_cache || !slot_mapping || !key_strides || !value_strides)
    return MVB_ERR_INVALID_ARGUMENT;
  return launch_reshape_and_cache(key, key_strides, value, value_strides, kv_cache, num_blocks,
                                  block_size, num_kv_heads, head_dim, slot_mapping, num_tokens, eb,
                                  status, static_cast<cudaStream_t>(stream));
}

size_t mvb_paged_attention_workspace_size(int64_t max_num_tokens, int64_t max_num_requests,
                                          int32_t num_q_heads, int32_t num_kv_heads,
                                          int32_t head_dim) {
  if (max_num_tokens < 0 || max_num_requests < 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      head_dim <= 0)
    return 0;
  return workspace_bytes_for(max_num_tokens, max_num_requests, num_q_heads, num_kv_heads,
                             head_dim);
}

int mvb_paged_attention(const void* query, int64_t query_token_stride, int64_t query_head_stride,
                        void* output, const void* kv_cache, int64_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, const int64_t* query_positions,
                        const int64_t* query_context_starts, const int64_t* query_start_locations,
                        const int64_t* context_lengths, const int64_t* block_table,
                        int64_t block_table_row_stride, int64_t block_table_width,
                        int64_t num_tokens, int64_t num_requests, int32_t num_q_heads, float scale,
                        int32_t dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                        void* stream) {
  if (elem_bytes_of(dtype) == 0) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens < 0 || num_requests < 0 || num_blocks < 0 || block_size <= 0 ||
      num_kv_heads <= 0 || head_dim <= 0 || num_q_heads <= 0 || block_table_width < 0)
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return MVB_ERR_UNSUPPORTED_SHAPE;
  if (num_tokens == 0) return MVB_OK;
  if (!query || !output || !kv_cache || !query_positions || !query_context_starts ||
      !query_start_locations || (num_requests > 0 && (!context_lengths || !block_table)))
    return MVB_ERR_INVALID_ARGUMENT;
  AttentionProblem p;
  p.query = query;
  p.q_st = query_token_stride;
  p.q_sh = query_head_stride;
  p.out = output;
  p.cache = kv_cache;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.qpos = query_positions;
  p.qstart = query_context_starts;
  p.qsl = query_start_locations;
  p.ctx_len = context_lengths;
  p.table = block_table;
  p.table_stride = block_table_row_stride;
  p.table_width = block_table_width;
  p.num_tokens = num_tokens;
  p.num_requests = num_requests;
  p.num_q_heads = num_q_heads;
  p.scale = scale;
  p.dtype = dtype;
  p.workspace = workspace;
  p.workspace_bytes = workspace_bytes;
  p.status = status;
  p.stream = static_cast<cudaStream_t>(stream);
  return run_paged_attention(p);
}

int mvb_attention_forward(const void* query, int64_t query_token_stride, int64_t query_head_stride,
                          const void* key, const int64_t* key_strides, const void* value,
                          const int64_t* value_strides, void* output, void* kv_cache,
                          int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                          int32_t head_dim, const int64_t* query_positions,
                          const int64_t* query_context_starts, const int64_t* query_start_locations,
                          const int64_t* context_lengths, const int64_t* block_table,
                          int64_t block_table_row_stride, int64_t block_table_width,
                          const int64_t* slot_mapping, int64_t num_tokens, int64_t num_requests,
                          int32_t num_q_heads, float scale, int32_t dtype, void* workspace,
                          size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = mvb_reshape_and_cache(key, key_strides, value, value_strides, kv_cache, num_blocks,
                                 block_size, num_kv_heads, head_dim, slot_mapping, num_tokens,
                                 dtype, status, stream);
  if (rc != MVB_OK) return rc;
  return mvb_paged_attention(query, query_token_stride, query_head_stride, output, kv_cache,
                             num_blocks, block_size, num_kv_heads, head_dim, query_positions,
                             query_context_starts, query_start_locations, context_lengths,
                             block_table, block_table_row_stride, block_table_width, num_tokens,
                             num_requests, num_q_heads, scale, dtype, workspace, workspace_bytes,
                             status, stream);
}

int mvb_qk_norm_rope_and_cache(const void* query, const int64_t* q_strides, const void* key,
                               const int64_t* k_strides, const void* value,
                               const int64_t* v_strides, void* q_out, const void* q_weight,
                               const void* k_weight, float eps, const float* inv_freq,
                               const int64_t* positions, void* kv_cache, int64_t num_blocks,
                               int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                               const int64_t* slot_mapping, int64_t num_tokens,
                               int32_t num_q_heads, int32_t dtype, int32_t* status, void* stream) {
  if (dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens < 0 || num_blocks < 0 || block_size <= 0 || num_kv_heads <= 0 ||
      num_q_heads <= 0 || head_dim <= 0 || !(eps >= 0.f))
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MVB_OK;
  if (!query || !key || !value || !q_out || !q_weight || !k_weight || !inv_freq || !positions ||
      !kv_cache || !slot_mapping || !q_strides || !k_strides || !v_strides)
    return MVB_ERR_INVALID_ARGUMENT;
  QkPrologueArgs a;
  a.query = query;
  a.q_strides = q_strides;
  a.key = key;
  a.k_strides = k_strides;
  a.value = value;
  a.v_strides = v_strides;
  a.q_out = q_out;
  a.q_weight = q_weight;
  a.k_weight = k_weight;
  a.eps = eps;
  a.inv_freq = inv_freq;
  a.positions = positions;
  a.kv_cache = kv_cache;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.slot_mapping = slot_mapping;
  a.num_tokens = num_tokens;
  a.num_q_heads = num_q_heads;
  a.dtype = dtype;
  a.status = status;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_qk_prologue(a);
}

int mvb_sample_with_noise(const void* logits, int64_t row_stride, int64_t num_rows, int64_t vocab,
                          int32_t dtype, const float* temperature, const int32_t* top_k,
                          const float* top_p, const uint64_t* seed, const int64_t* sample_index,
                          const float* noise, int64_t noise_row_stride, int64_t num_noise_rows,
                          const int32_t* noise_row, int64_t* out_tokens, void* stream) {
  if (elem_bytes_of(dtype) == 0) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_rows < 0 || vocab <= 0 || vocab >= ((int64_t)1 << 31) || row_stride < 0)
    return MVB_ERR_INVALID_ARGUMENT;
  if (noise != nullptr && (noise_row == nullptr || noise_row_stride < vocab || num_noise_rows < 0 ||
                           num_noise_rows > INT32_MAX))
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return MVB_OK;
  if (!logits || !temperature || !top_k || !top_p || !seed || !sample_index || !out_tokens)
    return MVB_ERR_INVALID_ARGUMENT;
  SampleArgs a;
  a.logits = logits;
  a.row_stride = row_stride;
  a.num_rows = num_rows;
  a.vocab = vocab;
  a.dtype = dtype;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.seed = seed;
  a.sample_index = sample_index;
  a.out_tokens = out_tokens;
  a.noise = num_noise_rows > 0 ? noise : nullptr;
  a.noise_stride = noise_row_stride;
  a.num_noise_rows = num_noise_rows;
  a.noise_row = noise_row;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_sample(a);
}

int mvb_sample(const void* logits, int64_t row_stride, int64_t num_rows, int64_t vocab,
               int32_t dtype, const float* temperature, const int32_t* top_k, const float* top_p,
               const uint64_t* seed, const int64_t* sample_index, int64_t* out_tokens,
               void* stream) {
  return mvb_sample_with_noise(logits, row_stride, num_rows, vocab, dtype, temperature, top_k, top_p,
                               seed, sample_index, nullptr, 0, 0, nullptr, out_tokens, stream);
}

int mvb_rms_norm(const void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
                 void* sum_out, void* out, const void* weight, float eps, int64_t num_rows, int32_t hidden,
                 int32_t dtype, void* stream) {
  if (dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_rows < 0 || hidden <= 0 || x_row_stride < hidden ||
      (residual != nullptr && (residual_row_stride < hidden || sum_out == nullptr)))
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return MVB_OK;
  if (!x || !out || !weight) return MVB_ERR_INVALID_ARGUMENT;
  RmsNormArgs a;
  a.x = x;
  a.x_stride = x_row_stride;
  a.residual = residual;
  a.r_stride = residual_row_stride;
  a.sum_out = sum_out;
  a.out = out;
  a.weight = weight;
  a.eps = eps;
  a.rows = num_rows;
  a.hidden = hidden;
  a.dtype = dtype;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_rms_norm(a);
}

int mvb_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t num_rows,
                 int32_t intermediate, int32_t dtype, void* stream) {
  if (dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_UNSUPPORTED_DTYPE;
  if (num_rows < 0 || intermediate <= 0 || gate_up_row_stride < 2 * (int64_t)intermediate)
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return MVB_OK;
  if (!gate_up || !out) return MVB_ERR_INVALID_ARGUMENT;
  SiluMulArgs a;
  a.gate_up = gate_up;
  a.gu_stride = gate_up_row_stride;
  a.out = out;
  a.rows = num_rows;
  a.inter = intermediate;
  a.dtype = dtype;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_silu_mul(a);
}

int mvb_build_metadata(const int32_t* num_computed_tokens, const int32_t* num_scheduled_tokens,
                       const int32_t* num_block_ids, const int32_t* block_ids,
                       const uint8_t* requires_sampling, const int32_t* input_token_ids,
                       int64_t num_requests, int64_t num_tokens, int64_t num_block_ids_total,
                       int64_t num_sampled, int64_t request_capacity, int64_t token_capacity,
                       int64_t table_width, int64_t table_stride, int32_t block_size,
                       int64_t null_block_id, int32_t spec_kind, int64_t spec_param,
                       int64_t* input_ids, int64_t* positions, int64_t* context_starts,
                       int64_t* query_start_locations, int64_t* context_lengths,
                       int64_t* block_table, int64_t* slot_mapping, int64_t* sampling_rows,
                       int32_t* status, void* stream) {
  const int64_t kLimit = (int64_t)1 << 31;
  if (num_requests < 0 || num_tokens < 0 || num_tokens >= kLimit || num_block_ids_total < 0 ||
      num_block_ids_total >= kLimit || num_sampled < 0 || num_sampled > num_requests ||
      request_capacity < num_requests || token_capacity < num_tokens || table_width < 0 ||
      block_size <= 0)
    return MVB_ERR_INVALID_ARGUMENT;
  if (spec_kind != MVB_SPEC_FULL && spec_kind != MVB_SPEC_SLIDING_WINDOW &&
      spec_kind != MVB_SPEC_CHUNKED_LOCAL)
    return MVB_ERR_INVALID_ARGUMENT;
  if (spec_kind != MVB_SPEC_FULL && spec_param <= 0) return MVB_ERR_INVALID_ARGUMENT;
  if (block_table && table_stride < table_width) return MVB_ERR_INVALID_ARGUMENT;
  if (num_requests > 0 && (!num_computed_tokens || !num_scheduled_tokens || !num_block_ids))
    return MVB_ERR_INVALID_ARGUMENT;
  if ((num_block_ids_total > 0 && !block_ids) || (num_sampled > 0 && !requires_sampling) ||
      (num_sampled > 0 && !sampling_rows) ||
      (input_ids && num_tokens > 0 && !input_token_ids))
    return MVB_ERR_INVALID_ARGUMENT;
  if (num_requests > kMaxMetadataRequests) return MVB_ERR_UNSUPPORTED_SHAPE;
  if (token_capacity == 0 && request_capacity == 0 && !query_start_locations) return MVB_OK;
  MetadataArgs a;
  a.num_computed = num_computed_tokens;
  a.num_scheduled = num_scheduled_tokens;
  a.num_block_ids = num_block_ids;
  a.block_ids = block_ids;
  a.requires_sampling = requires_sampling;
  a.input_token_ids = input_token_ids;
  a.num_requests = num_requests;
  a.num_tokens = num_tokens;
  a.num_block_ids_total = num_block_ids_total;
  a.num_sampled = num_sampled;
  a.request_capacity = request_capacity;
  a.token_capacity = token_capacity;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.block_size = block_size;
  a.null_block_id = null_block_id;
  a.spec_kind = spec_kind;
  a.spec_param = spec_param;
  a.input_ids = input_ids;
  a.positions = positions;
  a.context_starts = context_starts;
  a.query_start_locations = query_start_locations;
  a.context_lengths = context_lengths;
  a.block_table = block_table;
  a.slot_mapping = slot_mapping;
  a.sampling_rows = sampling_rows;
  a.status = status;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_build_metadata(a);
}

}  // extern "C"
