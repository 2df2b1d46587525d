/*
 * mvb200.h — C ABI of the B200 (sm_100a) paged-attention backend for
 * micro-vLLM.
 *
 * Every entry point takes plain device pointers, element strides, sizes and
 * a cudaStream_t passed as `void*`; none allocates memory, synchronises the
 * host or takes a torch type.  All work is enqueued on `stream`, so the
 * calls can be issued from any host language and captured in a CUDA graph
 * once the workspace exists.  Return value: MVB_OK or a negative MVB_ERR_*.
 *
 * Tensor layouts (element offsets, 64-bit everywhere):
 *   kv_cache   [2, num_blocks, block_size, num_kv_heads, head_dim], contiguous
 *              (plane 0 = keys, plane 1 = values) — the layout ModelRunner
 *              allocates (model_runner.py:678-703 in the reference project).
 *   query      [num_tokens, num_q_heads, head_dim], innermost stride 1.
 *   key/value  [num_tokens, num_kv_heads, head_dim], any strides.
 *   output     [num_tokens, num_q_heads, head_dim], contiguous.
 *   metadata   int64 device arrays with the meaning of the reference's
 *              AttentionMetadata (attention/attention.py:12-28).
 */
#ifndef MVB200_H
#define MVB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MVB_API __attribute__((visibility("default")))
#else
#define MVB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MVB_OK 0
#define MVB_ERR_INVALID_ARGUMENT (-1)   /* null pointer, negative size, bad stride   */
#define MVB_ERR_UNSUPPORTED_DTYPE (-2)  /* dtype not supported by this entry point  */
#define MVB_ERR_UNSUPPORTED_SHAPE (-3)  /* head ratio / head_dim outside the limits */
#define MVB_ERR_WORKSPACE_TOO_SMALL (-4)
#define MVB_ERR_CUDA (-5)               /* a CUDA call failed; see mvb_last_cuda_error */

/* Element types. */
#define MVB_DTYPE_F16 0
#define MVB_DTYPE_BF16 1
#define MVB_DTYPE_F32 2

/* Bits OR-ed into the optional device status word by the kernels. */
#define MVB_STATUS_SLOT_OUT_OF_RANGE 1   /* slot >= num_blocks*block_size: row skipped  */
#define MVB_STATUS_BLOCK_OUT_OF_RANGE 2  /* block id outside [0,num_blocks): key hidden */
#define MVB_STATUS_POSITION_PAST_TABLE 4 /* position past its request's block ids: slot -1 */
#define MVB_STATUS_INCONSISTENT_COUNTS 8 /* counts disagree with the sizes: padding only */
#define MVB_STATUS_WAIT_TIMEOUT 16       /* a kernel's bounded wait ran out: its rows are undefined */

/* Visibility specs of mvb_build_metadata (attention/spec.py). */
#define MVB_SPEC_FULL 0           /* FullAttentionSpec: start 0                          */
#define MVB_SPEC_SLIDING_WINDOW 1 /* SlidingWindowSpec(param): max(0, pos - param + 1)  */
#define MVB_SPEC_CHUNKED_LOCAL 2  /* ChunkedLocalSpec(param): (pos / param) * param     */

/* Library version, (major << 16) | minor. */
MVB_API int mvb_version(void);

/* Human-readable name of a status code. */
MVB_API const char* mvb_status_string(int status);

/* cudaError_t of the last failed CUDA call on this host thread (0 if none). */
MVB_API int mvb_last_cuda_error(void);

/*
 * KV-cache scatter ("reshape_and_cache").
 *
 * Replaces write_kv_cache (src/micro_vllm/attention/operators/reference.py:84-98)
 * and triton_write_kv_cache / _write_kv_cache_kernel
 * (src/micro_vllm/attention/operators/triton_paged.py:293-325, :11-68).
 *
 * For every token t and KV head h, copies key[t,h,:] to
 * kv_cache[0, s / block_size, s % block_size, h, :] and value[t,h,:] to
 * plane 1, where s = slot_mapping[t].  The copy is bit-exact.  A negative
 * slot writes nothing (CUDA-graph padding); a slot past the pool writes
 * nothing and sets MVB_STATUS_SLOT_OUT_OF_RANGE in *status when status is
 * not NULL.  key_strides / value_strides are element strides of
 * [token, head, dim] (host arrays of 3).  dtype is any MVB_DTYPE_*.
 */
MVB_API int mvb_reshape_and_cache(const void* key, const int64_t* key_strides, const void* value,
                          const int64_t* value_strides, void* kv_cache, int64_t num_blocks,
                          int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                          const int64_t* slot_mapping, int64_t num_tokens, int32_t dtype,
                          int32_t* status, void* stream);

/*
 * Bytes of device workspace mvb_paged_attention needs for batches of at
 * most max_num_tokens query tokens and max_num_requests requests.  The
 * workspace must be 256-byte aligned; its contents need no initialisation
 * and are owned by the library between calls on the same stream.
 */
MVB_API size_t mvb_paged_attention_workspace_size(int64_t max_num_tokens, int64_t max_num_requests,
                                          int32_t num_q_heads, int32_t num_kv_heads,
                                          int32_t head_dim);

/*
 * Paged attention over the cache (no cache write).
 *
 * Replaces the attention part of ReferenceAttentionOperator.forward
 * (src/micro_vllm/attention/operators/reference.py:26-81, with
 * gather_kv_cache :101-138) and triton_paged_attention /
 * _paged_attention_kernel (src/micro_vllm/attention/operators/triton_paged.py:328-389,
 * :97-290).
 *
 * Query token t of request r (query_start_locations[r] <= t <
 * query_start_locations[r+1]) attends to the logical key positions
 *   max(ctx_start[first token of r], ctx_start[t]) .. min(context_lengths[r]-1, pos[t])
 * read through block_table[r, p / block_size]; query head j uses KV head
 * j / (num_q_heads / num_kv_heads); weights are softmax(q.k * scale) in
 * fp32.  Rows of tokens owned by no request are written as 0.  fp16 and
 * bf16 run the tensor-core kernels; fp32 runs the exact CUDA-core kernel.
 */
MVB_API int mvb_paged_attention(const void* query, int64_t query_token_stride, int64_t query_head_stride,
                        void* output, const void* kv_cache, int64_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, const int64_t* query_positions,
                        const int64_t* query_context_starts, const int64_t* query_start_locations,
                        const int64_t* context_lengths, const int64_t* block_table,
                        int64_t block_table_row_stride, int64_t block_table_width,
                        int64_t num_tokens, int64_t num_requests, int32_t num_q_heads, float scale,
                        int32_t dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                        void* stream);

/*
 * One AttentionOperator.forward: mvb_reshape_and_cache of key/value at
 * slot_mapping, then mvb_paged_attention, on the same stream.
 *
 * Replaces AttentionOperator.forward (src/micro_vllm/attention/operators/base.py:30-40)
 * as implemented by ReferenceAttentionOperator (reference.py:14-81) and
 * TritonPagedAttentionOperator (triton_paged.py:392-418).
 */
MVB_API int mvb_attention_forward(const void* query, int64_t query_token_stride, int64_t query_head_stride,
                          const void* key, const int64_t* key_strides, const void* value,
                          const int64_t* value_strides, void* output, void* kv_cache,
                          int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                          int32_t head_dim, const int64_t* query_positions,
                          const int64_t* query_context_starts, const int64_t* query_start_locations,
                          const int64_t* context_lengths, const int64_t* block_table,
                          int64_t block_table_row_stride, int64_t block_table_width,
                          const int64_t* slot_mapping, int64_t num_tokens, int64_t num_requests,
                          int32_t num_q_heads, float scale, int32_t dtype, void* workspace,
                          size_t workspace_bytes, int32_t* status, void* stream);

/*
 * mvb_paged_attention for callers that cannot allocate device memory.
 *
 * No counterpart in the reference project: it exists for hosts that cannot
 * hand the library a workspace — a plugin host whose device memory belongs
 * to its own arena allocator and that forbids other allocations, a serving
 * loop that must not risk an allocation failing or blocking mid-run, or a
 * language binding with no access to CUDA memory management.
 *
 * Same arguments and results as mvb_paged_attention minus the workspace.
 * The scratch it needs lives in a 24 MiB region compiled into the library,
 * which every GPU that loads the library holds until the process exits.
 * Batches needing more (mvb_paged_attention_workspace_size above 24 MiB,
 * i.e. tens of thousands of requests on the tensor-core path) are rejected
 * with MVB_ERR_WORKSPACE_TOO_SMALL; the exact CUDA-core path (fp32, other
 * head sizes) needs no scratch and takes any batch.  The first call on each
 * device looks up the region's device address (cudaGetSymbolAddress with
 * that device current) and keeps it for the life of the process; make that
 * first call before any stream capture, and do not call this entry point
 * after cudaDeviceReset on that device (the kept address would be stale).
 * All calls share the
 * region: calls whose GPU work overlaps (different streams or host threads
 * on one device) race and must be serialised by the caller.
 */
MVB_API int mvb_paged_attention_no_alloc(const void* query, int64_t query_token_stride,
                                         int64_t query_head_stride, void* output,
                                         const void* kv_cache, int64_t num_blocks,
                                         int32_t block_size, int32_t num_kv_heads,
                                         int32_t head_dim, const int64_t* query_positions,
                                         const int64_t* query_context_starts,
                                         const int64_t* query_start_locations,
                                         const int64_t* context_lengths,
                                         const int64_t* block_table,
                                         int64_t block_table_row_stride,
                                         int64_t block_table_width, int64_t num_tokens,
                                         int64_t num_requests, int32_t num_q_heads, float scale,
                                         int32_t dtype, int32_t* status, void* stream);

/*
 * Test hook for the attention kernels' bounded waits (no counterpart in the
 * reference project).
 *
 * Arms a one-shot stall for the next paged-decode launch issued from the
 * calling host thread: the producer warp of decode CTA `cta` issues nothing
 * for the `tile`-th 16-token tile of its share (no copy is in flight for that
 * stage, so nothing is withheld from a copy in progress), and every mbarrier
 * wait of that launch gives up after `wait_limit` polls.  The consumers'
 * wait for the skipped tile runs out: the launch sets MVB_STATUS_WAIT_TIMEOUT
 * in its status word, lets the copies it issued land and returns, and the
 * context stays usable; rows of that launch are undefined.  The next launch
 * runs normally.  wait_limit <= 0 disarms.  Returns MVB_OK.
 */
MVB_API int mvb_debug_arm_decode_stall(int32_t cta, int32_t tile, int32_t wait_limit);

/*
 * Fused Qwen3 attention prologue: per-head RMSNorm of query and key, rotary
 * position embedding of both, and the KV-cache write — one launch.
 *
 * Replaces, in one call, what Qwen3Attention.forward does between the
 * projections and the attention operator (src/micro_vllm/models/qwen.py:89-91):
 * q_norm / k_norm (RMSNorm.forward, src/micro_vllm/layers/normalization.py:15-22),
 * RotaryEmbedding.forward (src/micro_vllm/layers/rotary_embedding.py:22-52),
 * and the operator's first step write_kv_cache
 * (src/micro_vllm/attention/operators/reference.py:84-98).
 *
 * query [T, Hq, 128], key / value [T, Hkv, 128]: element strides
 * q/k/v_strides[3] (host arrays), unit innermost stride, rows 8-byte
 * aligned.  q_out [T, Hq, 128] contiguous receives the normalised, rotated
 * query; kv_cache plane 0 receives the normalised, rotated key and plane 1
 * the value at slot_mapping[t] (negative slot: nothing; past the pool:
 * nothing and MVB_STATUS_SLOT_OUT_OF_RANGE).  q_weight / k_weight [128] are
 * the RMSNorm weights in the activation dtype; inv_freq [64] (fp32) the
 * rotary inverse frequencies 1 / base^(2i/128) evaluated by the caller as the
 * reference does; positions [T] int64.  dtype MVB_DTYPE_F16 or _BF16.
 * head_dim must be 128 (else MVB_ERR_UNSUPPORTED_SHAPE).
 */
MVB_API int mvb_qk_norm_rope_and_cache(const void* query, const int64_t* q_strides,
                                       const void* key, const int64_t* k_strides,
                                       const void* value, const int64_t* v_strides, void* q_out,
                                       const void* q_weight, const void* k_weight, float eps,
                                       const float* inv_freq, const int64_t* positions,
                                       void* kv_cache, int64_t num_blocks, int32_t block_size,
                                       int32_t num_kv_heads, int32_t head_dim,
                                       const int64_t* slot_mapping, int64_t num_tokens,
                                       int32_t num_q_heads, int32_t dtype, int32_t* status,
                                       void* stream);

/*
 * Batched token sampler: the next token of every logits row in one launch.
 *
 * Replaces the per-row loop of Sampler.__call__ / _sample_row with
 * _apply_top_k and _apply_top_p (src/micro_vllm/sampling/sampler.py:14-87),
 * which synchronises the host once per row.
 *
 * logits [num_rows, vocab] with row stride row_stride (elements, >= 0: rows
 * may repeat), any MVB_DTYPE_*.  Per row (device arrays of num_rows): temperature (0 =
 * greedy: the first index of the largest logit, as torch.argmax), top_k (<= 0
 * or >= vocab: no filter), top_p (1 = no filter), seed and sample_index.
 * A stochastic row keeps the top_k largest of x = logit / temperature
 * (equal values at the cut: lowest indices first; division by T > 0 is
 * monotone, so tokens are ordered by the logit, which also orders equal x
 * from different fp32 logits), then, in descending order, every token whose
 * mass before it is <= top_p (masses exp(x - max) in 1.31 fixed point, so a
 * token below 2^-31 of the max has none and sits below any top-p cut), and
 * draws one token in proportion to its mass with a uniform number from
 * Philox4x32-10 keyed by seed with sample_index as the counter (the same pair
 * always gives the same token; the stream differs from torch's generator).
 * out_tokens (device int64 [num_rows]) receives the token ids.  Nothing is
 * allocated and the host is not synchronised.
 */
MVB_API int mvb_sample(const void* logits, int64_t row_stride, int64_t num_rows, int64_t vocab,
                       int32_t dtype, const float* temperature, const int32_t* top_k,
                       const float* top_p, const uint64_t* seed, const int64_t* sample_index,
                       int64_t* out_tokens, void* stream);

/*
 * mvb_sample with the reference's random stream for chosen rows.
 *
 * torch.multinomial(probabilities, 1, generator), as the reference's
 * _sample_row calls it (src/micro_vllm/sampling/sampler.py:52-61), picks the
 * token that maximises probability / q, q = torch.empty_like(probabilities)
 * .exponential_(1, generator) — an exponential race.  A row r with
 * 0 <= noise_row[r] < num_noise_rows takes that race over its kept set with
 * q = noise + noise_row[r] * noise_row_stride (float32, vocab values, drawn
 * by the caller from a generator seeded as the reference seeds it); the
 * probability is exp(x - max x), x = logit / temperature in fp32 (the
 * softmax denominator is common to all tokens), so the token is the
 * reference's unless its two best ratios agree to within fp32 rounding.
 * Other rows draw as mvb_sample.  noise may be NULL (every row draws as
 * mvb_sample); otherwise noise_row (device int32 [num_rows]) must be given
 * and noise_row_stride >= vocab.  Greedy rows ignore their noise row.
 */
MVB_API int mvb_sample_with_noise(const void* logits, int64_t row_stride, int64_t num_rows,
                                  int64_t vocab, int32_t dtype, const float* temperature,
                                  const int32_t* top_k, const float* top_p, const uint64_t* seed,
                                  const int64_t* sample_index, const float* noise,
                                  int64_t noise_row_stride, int64_t num_noise_rows,
                                  const int32_t* noise_row, int64_t* out_tokens, void* stream);

/*
 * RMSNorm of a Qwen3 decoder layer, optionally after its residual add, in
 * one launch (the reference model runs each as a chain of torch kernels).
 *
 * Replaces RMSNorm.forward (src/micro_vllm/layers/normalization.py:15-22)
 * and, with residual, the `residual + hidden_states` before it
 * (src/micro_vllm/models/qwen.py:151-154).  x [num_rows, hidden] with row
 * stride x_row_stride (elements), unit column stride; weight [hidden]; all
 * of dtype (MVB_DTYPE_F16 or _BF16).  With residual (same layout, its own
 * row stride) the row is h = x + residual rounded to dtype, written to
 * sum_out [num_rows, hidden] contiguous; without it h = x.  out [num_rows,
 * hidden] contiguous receives weight * dtype(h * 1/sqrt(mean(h^2) + eps)),
 * the statistics in fp32.  hidden and both row strides must be multiples of
 * 8 and the pointers 16-byte aligned (else MVB_ERR_UNSUPPORTED_SHAPE).
 */
MVB_API int mvb_rms_norm(const void* x, int64_t x_row_stride, const void* residual,
                         int64_t residual_row_stride, void* sum_out, void* out, const void* weight,
                         float eps, int64_t num_rows, int32_t hidden, int32_t dtype, void* stream);

/*
 * silu(gate) * up of a SwiGLU MLP in one launch.
 *
 * Replaces `F.silu(gate_proj(h))` times `up_proj(h)` in SwiGLUMLP.forward
 * (src/micro_vllm/layers/mlp.py:19-21) for one projection that computes both:
 * gate_up [num_rows, >= 2 * intermediate] with row stride gate_up_row_stride
 * holds the gate columns then the up columns.  out [num_rows, intermediate]
 * contiguous receives dtype(dtype(silu(gate)) * up), silu in fp32.
 * intermediate and the row stride must be multiples of 8 and the pointers
 * 16-byte aligned.
 */
MVB_API int mvb_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out,
                         int64_t num_rows, int32_t intermediate, int32_t dtype, void* stream);

/*
 * Device-side build of one step's attention metadata (one cache group).
 *
 * Replaces the host loops of ModelRunner._flatten_model_input,
 * _build_slot_mapping and _build_block_table
 * (src/micro_vllm/worker/model_runner.py:751-900), the per-position loop of
 * Attention.build_metadata (src/micro_vllm/attention/attention.py:56-85) and
 * map_cache_slots (attention.py:31-41); with capacities above the actual
 * sizes it also pads as _CudaGraphExecution.copy_input does
 * (model_runner.py:78-122).
 *
 * Inputs (device, per scheduled request in plan order, num_requests of them):
 * num_computed_tokens, num_scheduled_tokens, num_block_ids (int32), the
 * requests' block ids concatenated (int32, num_block_ids_total of them),
 * requires_sampling (uint8, may be NULL when num_sampled is 0) and the
 * concatenated input token ids (int32 [num_tokens], may be NULL when
 * input_ids is NULL).  num_tokens, num_block_ids_total and num_sampled are
 * the sums of the counts, below 2^31; num_requests <= 16384 (else
 * MVB_ERR_UNSUPPORTED_SHAPE).
 *
 * Outputs (device int64, each may be NULL to skip it):
 *   input_ids, positions, context_starts, slot_mapping [token_capacity]
 *     (0, 0, 0, -1 past num_tokens); context_starts follow spec_kind /
 *     spec_param (MVB_SPEC_*);
 *   query_start_locations [request_capacity + 1] (num_tokens past
 *     num_requests + 1), context_lengths [request_capacity] (0 past
 *     num_requests);
 *   block_table [request_capacity, table_width], row stride table_stride,
 *     null_block_id past each request's block ids;
 *   sampling_rows [num_sampled]: the last token of each request with
 *     requires_sampling set.
 * A position whose logical block lies past its request's block ids (the
 * reference raises IndexError) gets slot -1 and sets
 * MVB_STATUS_POSITION_PAST_TABLE; counts that are negative, do not sum to
 * the sizes passed or exceed table_width leave padding only and set
 * MVB_STATUS_INCONSISTENT_COUNTS.  One launch; the host is not synchronised.
 */
MVB_API int mvb_build_metadata(const int32_t* num_computed_tokens,
                               const int32_t* num_scheduled_tokens, const int32_t* num_block_ids,
                               const int32_t* block_ids, const uint8_t* requires_sampling,
                               const int32_t* input_token_ids, int64_t num_requests,
                               int64_t num_tokens, int64_t num_block_ids_total,
                               int64_t num_sampled, int64_t request_capacity,
                               int64_t token_capacity, int64_t table_width, int64_t table_stride,
                               int32_t block_size, int64_t null_block_id, int32_t spec_kind,
                               int64_t spec_param, int64_t* input_ids, int64_t* positions,
                               int64_t* context_starts, int64_t* query_start_locations,
                               int64_t* context_lengths, int64_t* block_table,
                               int64_t* slot_mapping, int64_t* sampling_rows, int32_t* status,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MVB200_H */
