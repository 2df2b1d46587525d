// Shared device helpers for the B200 paged-attention kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mvb200.h"

namespace mvb {

// Records the CUDA error of the last failed call on this host thread.
void set_last_cuda_error(cudaError_t err);

// Returns MVB_OK, or MVB_ERR_CUDA after recording the pending launch error.
int check_launch();

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Index of the request owning flattened query token `t`: the largest r in
// [0, R) with qsl[r] <= t, or -1 when t lies in no request (t >= qsl[R],
// or every request before t is empty).  Zero-length requests (qsl[r] ==
// qsl[r+1], CUDA-graph padding) are skipped because a later request with the
// same start also satisfies qsl[r] <= t.  A negative start (malformed
// metadata) also yields -1, so callers may index qstart[qsl[r]] safely.
__device__ __forceinline__ int64_t find_request(const int64_t* __restrict__ qsl, int64_t R,
                                                int64_t t) {
  int64_t lo = 0, hi = R;  // answer in [lo-1, hi-1]
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (__ldg(qsl + mid) <= t)
      lo = mid + 1;
    else
      hi = mid;
  }
  int64_t r = lo - 1;
  if (r < 0 || t >= __ldg(qsl + r + 1) || __ldg(qsl + r) < 0) return -1;
  return r;
}

// Programmatic dependent launch (sm_90+): a kernel launched with
// programmatic stream serialization may start while the kernel before it in
// the stream still runs; grid_dependency_wait() returns once that kernel has
// completed and its writes are visible (at once for a normal launch), and
// allow_dependent_launch() lets the next such kernel start early.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

}  // namespace mvb
