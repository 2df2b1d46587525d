// reshape_and_cache: scatter the step's new K/V rows into the paged cache.
//
// Behaviour of write_kv_cache (reference.py:84-98 in the reference project)
// with the Triton backend's skip of negative slots (triton_paged.py:37-39).
// The work is a pure byte copy, bound by HBM: every (token, kv head) row of
// head_dim elements is read once from key/value and written once into plane
// 0/1 of the cache.  Rows are moved as 16-byte vectors when both sides allow
// it (dim stride 1, 16-byte aligned rows), otherwise element by element.
#include "mvb_common.cuh"

namespace mvb {
namespace {

// One thread per 16-byte vector of one row; grid-stride over
// num_tokens * num_kv_heads * vecs_per_row.
__global__ void __launch_bounds__(256) scatter_rows_vec16(
    const char* __restrict__ key, int64_t k_st, int64_t k_sh,  // byte strides
    const char* __restrict__ value, int64_t v_st, int64_t v_sh, char* __restrict__ cache,
    int64_t plane_bytes, int64_t num_slots, int32_t num_kv_heads, int32_t row_bytes,
    const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int32_t* status) {
  const int32_t vecs_per_row = row_bytes >> 4;
  const int64_t total = num_tokens * num_kv_heads * vecs_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t vec = (int32_t)(i % vecs_per_row);
    const int64_t row = i / vecs_per_row;
    const int32_t h = (int32_t)(row % num_kv_heads);
    const int64_t t = row / num_kv_heads;
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (status != nullptr && vec == 0 && h == 0) atomicOr(status, MVB_STATUS_SLOT_OUT_OF_RANGE);
      continue;
    }
    const int64_t dst = (slot * num_kv_heads + h) * (int64_t)row_bytes + ((int64_t)vec << 4);
    const uint4 kv = __ldg(reinterpret_cast<const uint4*>(key + t * k_st + h * k_sh) + vec);
    const uint4 vv = __ldg(reinterpret_cast<const uint4*>(value + t * v_st + h * v_sh) + vec);
    *reinterpret_cast<uint4*>(cache + dst) = kv;
    *reinterpret_cast<uint4*>(cache + plane_bytes + dst) = vv;
  }
}

// Element-wise fallback for strided or unaligned inputs; Elem is an
// unsigned integer of the element size so the copy is bit-exact.
template <typename Elem>
__global__ void __launch_bounds__(256) scatter_rows_elem(
    const Elem* __restrict__ key, int64_t k_st, int64_t k_sh, int64_t k_sd,
    const Elem* __restrict__ value, int64_t v_st, int64_t v_sh, int64_t v_sd,
    Elem* __restrict__ cache, int64_t plane_elems, int64_t num_slots, int32_t num_kv_heads,
    int32_t head_dim, const int64_t* __restrict__ slot_mapping, int64_t num_tokens,
    int32_t* status) {
  const int64_t total = num_tokens * num_kv_heads * head_dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t d = (int32_t)(i % head_dim);
    const int64_t row = i / head_dim;
    const int32_t h = (int32_t)(row % num_kv_heads);
    const int64_t t = row / num_kv_heads;
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (status != nullptr && d == 0 && h == 0) atomicOr(status, MVB_STATUS_SLOT_OUT_OF_RANGE);
      continue;
    }
    const int64_t dst = (slot * num_kv_heads + h) * head_dim + d;
    cache[dst] = key[t * k_st + h * k_sh + d * k_sd];
    cache[plane_elems + dst] = value[t * v_st + h * v_sh + d * v_sd];
  }
}

inline int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  // 148 SMs x 8 resident 256-thread CTAs covers the GPU; more adds nothing.
  const int64_t cap = 148 * 8 * 4;
  return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

int launch_reshape_and_cache(const void* key, const int64_t* ks, const void* value,
                             const int64_t* vs, void* kv_cache, int64_t num_blocks,
                             int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                             const int64_t* slot_mapping, int64_t num_tokens, int32_t elem_bytes,
                             int32_t* status, cudaStream_t stream) {
  if (num_tokens == 0) return MVB_OK;
  const int64_t num_slots = num_blocks * block_size;
  const int64_t plane_elems = num_slots * num_kv_heads * head_dim;
  const int32_t row_bytes = head_dim * elem_bytes;
  const bool vec_ok = ks[2] == 1 && vs[2] == 1 && (row_bytes % 16) == 0 &&
                      ((uintptr_t)key % 16) == 0 && ((uintptr_t)value % 16) == 0 &&
                      ((uintptr_t)kv_cache % 16) == 0 && ((ks[0] * elem_bytes) % 16) == 0 &&
                      ((ks[1] * elem_bytes) % 16) == 0 && ((vs[0] * elem_bytes) % 16) == 0 &&
                      ((vs[1] * elem_bytes) % 16) == 0;
  if (vec_ok) {
    const int64_t work = num_tokens * num_kv_heads * (row_bytes / 16);
    scatter_rows_vec16<<<grid_for(work, 256), 256, 0, stream>>>(
        static_cast<const char*>(key), ks[0] * elem_bytes, ks[1] * elem_bytes,
        static_cast<const char*>(value), vs[0] * elem_bytes, vs[1] * elem_bytes,
        static_cast<char*>(kv_cache), plane_elems * elem_bytes, num_slots, num_kv_heads, row_bytes,
        slot_mapping, num_tokens, status);
    return check_launch();
  }
  const int64_t work = num_tokens * num_kv_heads * head_dim;
  if (elem_bytes == 2) {
    scatter_rows_elem<uint16_t><<<grid_for(work, 256), 256, 0, stream>>>(
        static_cast<const uint16_t*>(key), ks[0], ks[1], ks[2],
        static_cast<const uint16_t*>(value), vs[0], vs[1], vs[2], static_cast<uint16_t*>(kv_cache),
        plane_elems, num_slots, num_kv_heads, head_dim, slot_mapping, num_tokens, status);
  } else {
    scatter_rows_elem<uint32_t><<<grid_for(work, 256), 256, 0, stream>>>(
        static_cast<const uint32_t*>(key), ks[0], ks[1], ks[2],
        static_cast<const uint32_t*>(value), vs[0], vs[1], vs[2], static_cast<uint32_t*>(kv_cache),
        plane_elems, num_slots, num_kv_heads, head_dim, slot_mapping, num_tokens, status);
  }
  return check_launch();
}

}  // namespace mvb
