// mvb_paged_attention_no_alloc: paged attention for callers that cannot
// allocate device memory.
//
// mvb_paged_attention needs a caller-provided workspace (planner arrays and
// the fp32 partials of requests split across CTAs).  Some hosts cannot
// provide one: a plugin host whose device memory is owned by its own arena
// allocator and that forbids other allocations, a latency-critical serving
// loop that must not risk an allocation failing or blocking mid-run, or a
// binding from a language with no handle on CUDA memory management.  This
// entry point uses a scratch region compiled into the library instead: a
// file-scope __device__ array of kNoAllocScratchBytes (24 MiB) that every GPU
// which loads the library holds until the process exits.
//
// On the host the array's name is only a stand-in, not a device address, so
// the first call on each device looks up the array's real device address
// with cudaGetSymbolAddress (with that device current) and caches it for the
// life of the process.  That first call should come before any stream
// capture.  The cached address belongs to the device's primary context:
// after cudaDeviceReset, or once the primary context has been released and
// created again, it is stale and this entry point must not be called.
// Every call shares the same region and leaves its contents behind; the kernels re-derive
// everything they read from it on each call (the planner rewrites its arrays
// and zeroes the merge counters and the zero row before the decode kernel
// starts), so no state carries over.  Two calls whose work overlaps on the
// GPU — on different streams, or on different host threads using the same
// device — race on the region and must be serialised by the caller.
#include <mutex>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)24 << 20;

static __device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

void* g_scratch_device_ptr[mvb::kMaxDevices] = {};
std::mutex g_scratch_mutex;

}  // namespace

extern "C" MVB_API int mvb_paged_attention_no_alloc(
    const void* query, int64_t query_token_stride, int64_t query_head_stride, void* output,
    const void* kv_cache, int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
    int32_t head_dim, const int64_t* query_positions, const int64_t* query_context_starts,
    const int64_t* query_start_locations, const int64_t* context_lengths,
    const int64_t* block_table, int64_t block_table_row_stride, int64_t block_table_width,
    int64_t num_tokens, int64_t num_requests, int32_t num_q_heads, float scale, int32_t dtype,
    int32_t* status, void* stream) {
  // Arguments are checked, and the batch is measured against the region, by
  // mvb_paged_attention itself: the tensor-core path lays out its workspace in
  // the region and answers MVB_ERR_WORKSPACE_TOO_SMALL when the batch needs
  // more than kNoAllocScratchBytes; the exact CUDA-core path (fp32, other head
  // sizes, unaligned views) uses no workspace and takes any batch.
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    mvb::set_last_cuda_error(err);
    return MVB_ERR_CUDA;
  }
  if (device < 0 || device >= mvb::kMaxDevices) return MVB_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_device_ptr[device] == nullptr) {
      void* ptr = nullptr;
      err = cudaGetSymbolAddress(&ptr, g_no_alloc_scratch);
      if (err != cudaSuccess) {
        mvb::set_last_cuda_error(err);
        return MVB_ERR_CUDA;
      }
      g_scratch_device_ptr[device] = ptr;
    }
    scratch = g_scratch_device_ptr[device];
  }
  return mvb_paged_attention(query, query_token_stride, query_head_stride, output, kv_cache,
                             num_blocks, block_size, num_kv_heads, head_dim, query_positions,
                             query_context_starts, query_start_locations, context_lengths,
                             block_table, block_table_row_stride, block_table_width, num_tokens,
                             num_requests, num_q_heads, scale, dtype, scratch,
                             kNoAllocScratchBytes, status, stream);
}
