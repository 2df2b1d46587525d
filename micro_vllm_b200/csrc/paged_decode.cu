// Split-KV GQA paged decode for head_dim 128, fp16/bf16, on tensor cores.
//
// Work item = (request, split of its KV positions, KV head), as produced by
// the device planner (plan.cu).  The kernel is persistent: each 128-thread
// CTA pulls items from an atomic cursor until none are left.
//
// Inside an item the four warps take 16-token tiles round-robin and run as
// independent flash-decoding lanes:
//   * staging: each warp streams its own K and V tiles (16 tokens x 256 B
//     per plane) into a private STAGES-deep shared-memory ring with 16-byte
//     cp.async.cg copies, one instruction covering two 256-byte token rows.
//     Rows are resolved through the block table per tile (one lookup when a
//     page holds >= 16 tokens).  The 16-byte chunk index is XOR-swizzled by
//     the row so ldmatrix reads are bank-conflict free.
//   * scores: S^T = K . Q^T with mma.sync m16n8k16 — the 16 tokens of the
//     tile are the M dimension and the N = 8 columns hold the queries of
//     the GQA group (query_len x group <= 8), so one K tile load serves
//     every query head that shares the KV head.
//   * softmax: fp32 online softmax per column; the column max is a 3-step
//     warp shuffle over the 8 lanes holding that column; sums are kept per
//     lane and reduced once at the end.
//   * P.V: O^T += V^T . P^T with the probabilities moved from the score
//     accumulator layout into the B-operand layout by movmatrix.trans.
// The four warps' (max, sum, O) states are merged through shared memory.
// A request with one split writes its output directly; otherwise each split
// stores an fp32 partial (O, max, sum) and the CTA that finishes last (an
// atomic count per request and KV head — no waiting) merges them.
//
// Semantics follow ReferenceAttentionOperator.forward (reference.py:14-81):
// query token t of request r sees positions
//   max(ctx_start[first token of r], ctx_start[t]) .. min(ctx_len[r]-1, pos[t]);
// softmax(q.k * scale) in fp32; empty gathered history -> 0, empty window
// -> NaN.  HBM traffic per item is one read of its K/V rows: the roofline
// is HBM bandwidth.
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRowBytes = kDecodeHeadDim * 2;   // one token's head row
constexpr int kTileTokens = 16;
constexpr int kTileBytes = kTileTokens * kRowBytes;  // 4 KiB per plane
constexpr int kStageBytes = 2 * kTileBytes;          // K + V
constexpr int kColStride = kDecodeHeadDim + 4;       // padded fp32 row in the merge buffer

struct DecodeParams {
  const char* query;
  int64_t q_st_bytes, q_sh_bytes;
  char* out;
  const char* cache;
  int64_t plane_bytes;
  int64_t num_blocks;
  int32_t block_size, bs_shift, num_kv_heads, group, num_q_heads;
  const int64_t *qpos, *qstart, *qsl, *ctx_len, *table;
  int64_t table_stride, table_width, num_requests;
  float scale_log2;
  const int32_t* ctrl;
  int32_t* cursor;
  const int32_t* unit_prefix;
  int32_t* merge_count;
  float* partial_o;    // [items][8][128]
  float2* partial_ml;  // [items][8]  (max, sum)
  int32_t* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  const int src_size = valid ? 16 : 0;  // 0 = zero-fill, nothing read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_size)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Physical block of logical position `pos` of a request, or -1 when the
// table has no valid entry for it.
__device__ __forceinline__ int64_t page_of(const DecodeParams& p, const int64_t* trow, int64_t pos,
                                           int64_t* offset) {
  int64_t lb;
  if (p.bs_shift >= 0) {
    lb = pos >> p.bs_shift;
    *offset = pos & (p.block_size - 1);
  } else {
    lb = pos / p.block_size;
    *offset = pos - lb * p.block_size;
  }
  if (lb < 0 || lb >= p.table_width) return -1;
  const int64_t blk = __ldg(trow + lb);
  return (blk >= 0 && blk < p.num_blocks) ? blk : -1;
}

template <typename T, int STAGES>
__global__ void __launch_bounds__(kThreads) paged_decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_item;
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int num_items = p.ctrl[kCtrlNumItems];
  const int64_t chunk = p.ctrl[kCtrlChunk];
  const uint32_t wbase = smem_u32(smem + warp * STAGES * kStageBytes);
  const int64_t row_stride = (int64_t)p.num_kv_heads * kRowBytes;  // bytes between slots

  for (;;) {
    if (threadIdx.x == 0) s_item = atomicAdd(p.cursor, 1);
    __syncthreads();
    const int item = s_item;
    if (item >= num_items) break;

    // ---- locate the item ----
    const int h = item % p.num_kv_heads;
    const int64_t unit = item / p.num_kv_heads;
    int64_t lo_i = 0, hi_i = p.num_requests;  // largest r with unit_prefix[r] <= unit
    while (lo_i < hi_i) {
      const int64_t mid = (lo_i + hi_i) >> 1;
      if (__ldg(p.unit_prefix + mid) <= unit)
        lo_i = mid + 1;
      else
        hi_i = mid;
    }
    const int64_t r = lo_i - 1;
    const int64_t u0 = __ldg(p.unit_prefix + r);
    const int split = (int)(unit - u0);
    const int nsplit = (int)(__ldg(p.unit_prefix + r + 1) - u0);
    const int64_t qs = __ldg(p.qsl + r);
    const int ncols = (int)(__ldg(p.qsl + r + 1) - qs) * p.group;
    const int64_t lo_r = max(__ldg(p.qstart + qs), (int64_t)0);
    const int64_t hi_r = __ldg(p.ctx_len + r);
    const bool empty_history = hi_r <= lo_r;
    const int64_t tile0 = (lo_r & ~(int64_t)15) + (int64_t)split * chunk;
    const int64_t kv_begin = max(tile0, lo_r);
    const int64_t kv_end = min(tile0 + chunk, hi_r);
    const int ntiles = kv_end > kv_begin ? (int)((kv_end - tile0 + 15) >> 4) : 0;
    const int64_t* trow = p.table + r * p.table_stride;

    // Visible window of this lane's two columns (2c, 2c+1).
    int64_t wlo[2], whi[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = 2 * c + j;
      if (n < ncols) {
        const int64_t t = qs + n / p.group;
        wlo[j] = max(lo_r, __ldg(p.qstart + t));
        whi[j] = min(hi_r - 1, __ldg(p.qpos + t));
      } else {
        wlo[j] = 1;
        whi[j] = 0;
      }
    }
    // Q^T as B fragments: column g = (query g / group, head g % group).
    uint32_t qb[8][2];
    if (g < ncols) {
      const int64_t t = qs + g / p.group;
      const int hq = h * p.group + g % p.group;
      const char* qrow = p.query + t * p.q_st_bytes + (int64_t)hq * p.q_sh_bytes;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qb[ks][0] = __ldg(reinterpret_cast<const uint32_t*>(qrow + (16 * ks + 2 * c) * 2));
        qb[ks][1] = __ldg(reinterpret_cast<const uint32_t*>(qrow + (16 * ks + 2 * c + 8) * 2));
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) qb[ks][0] = qb[ks][1] = 0u;
    }

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    const int nt = ntiles > warp ? (ntiles - 1 - warp) / kWarps + 1 : 0;
    const bool one_page_per_tile = p.bs_shift >= 4;

    // Issue the cp.async copies of local tile i into ring slot i % STAGES.
    auto issue = [&](int i) {
      const int64_t tstart = tile0 + (int64_t)(warp + kWarps * i) * kTileTokens;
      const uint32_t kdst = wbase + (i % STAGES) * kStageBytes;
      const int ch = lane & 15;
      int64_t off0 = 0, blk0 = -1;
      if (one_page_per_tile) blk0 = page_of(p, trow, tstart, &off0);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int row = 2 * jj + (lane >> 4);
        const int64_t pos = tstart + row;
        int64_t blk, off;
        if (one_page_per_tile) {
          blk = blk0;
          off = off0 + row;
        } else {
          blk = page_of(p, trow, pos, &off);
        }
        const bool valid = blk >= 0 && pos >= kv_begin && pos < kv_end;
        const char* src =
            valid ? p.cache + (blk * p.block_size + off) * row_stride + (int64_t)h * kRowBytes + ch * 16
                  : p.cache;
        const uint32_t dst = kdst + row * kRowBytes + ((ch ^ (row & 7)) << 4);
        cp_async_16(dst, src, valid);
        cp_async_16(dst + kTileBytes, src + p.plane_bytes * valid, valid);
      }
    };

#pragma unroll
    for (int i = 0; i < STAGES - 1; ++i) {
      if (i < nt) issue(i);
      cp_async_commit();
    }
    for (int i = 0; i < nt; ++i) {
      cp_async_wait<STAGES - 2>();
      __syncwarp();
      if (i + STAGES - 1 < nt) issue(i + STAGES - 1);
      cp_async_commit();

      const uint32_t kb = wbase + (i % STAGES) * kStageBytes;
      const uint32_t vb = kb + kTileBytes;
      const int64_t tstart = tile0 + (int64_t)(warp + kWarps * i) * kTileTokens;

      float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * ks + (lane >> 4);
        uint32_t a[4];
        ldsm_x4(kb + row * kRowBytes + ((ch ^ (row & 7)) << 4), a);
        mma16816<T>(s, a, qb[ks][0], qb[ks][1]);
      }

      // Mask: token rows g and g+8 of the tile, columns 2c and 2c+1.
      const int64_t p0 = tstart + g, p1 = p0 + 8;
      const bool in0 = p0 >= kv_begin && p0 < kv_end, in1 = p1 >= kv_begin && p1 < kv_end;
      bool ok0, ok1;
      {
        int64_t off;
        if (one_page_per_tile) {
          const bool page_ok = page_of(p, trow, tstart, &off) >= 0;
          ok0 = in0 && page_ok;
          ok1 = in1 && page_ok;
        } else {
          ok0 = in0 && page_of(p, trow, p0, &off) >= 0;
          ok1 = in1 && page_of(p, trow, p1, &off) >= 0;
        }
        if (p.status != nullptr && (ok0 != in0 || ok1 != in1))
          atomicOr(p.status, MVB_STATUS_BLOCK_OUT_OF_RANGE);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        s[j] = (ok0 && p0 >= wlo[j] && p0 <= whi[j]) ? s[j] * p.scale_log2 : -INFINITY;
        s[2 + j] = (ok1 && p1 >= wlo[j] && p1 <= whi[j]) ? s[2 + j] * p.scale_log2 : -INFINITY;
      }
      float corr[2], pr[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float tmax = fmaxf(s[j], s[2 + j]);
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
        const float mn = fmaxf(m[j], tmax);
        const float mu = mn == -INFINITY ? 0.f : mn;
        corr[j] = exp2f(m[j] - mu);
        pr[j] = exp2f(s[j] - mu);
        pr[2 + j] = exp2f(s[2 + j] - mu);
        l[j] = l[j] * corr[j] + pr[j] + pr[2 + j];
        m[j] = mn;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= corr[0];
        o[mt][1] *= corr[1];
        o[mt][2] *= corr[0];
        o[mt][3] *= corr[1];
      }
      const uint32_t pb0 = movmatrix_t(pack2<T>(pr[0], pr[1]));
      const uint32_t pb1 = movmatrix_t(pack2<T>(pr[2], pr[3]));
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int row = (lane & 7) + (lane >> 4) * 8;
        const int ch = 2 * mt + ((lane >> 3) & 1);
        uint32_t a[4];
        ldsm_x4_t(vb + row * kRowBytes + ((ch ^ (row & 7)) << 4), a);
        mma16816<T>(o[mt], a, pb0, pb1);
      }
    }
    cp_async_wait<0>();

    // ---- merge the four warps ----
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l[j] += __shfl_xor_sync(0xffffffffu, l[j], 4);
      l[j] += __shfl_xor_sync(0xffffffffu, l[j], 8);
      l[j] += __shfl_xor_sync(0xffffffffu, l[j], 16);
    }
    __syncthreads();  // every warp is done with its ring: reuse it
    float* so = reinterpret_cast<float*>(smem);             // [warp][col][kColStride]
    float2* sml = reinterpret_cast<float2*>(so + kWarps * kDecodeCols * kColStride);  // [warp][col]
    {
      float* mine = so + warp * kDecodeCols * kColStride;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        mine[(2 * c) * kColStride + 16 * mt + g] = o[mt][0];
        mine[(2 * c + 1) * kColStride + 16 * mt + g] = o[mt][1];
        mine[(2 * c) * kColStride + 16 * mt + g + 8] = o[mt][2];
        mine[(2 * c + 1) * kColStride + 16 * mt + g + 8] = o[mt][3];
      }
      if (g == 0) {
        sml[warp * kDecodeCols + 2 * c] = make_float2(m[0], l[0]);
        sml[warp * kDecodeCols + 2 * c + 1] = make_float2(m[1], l[1]);
      }
    }
    __syncthreads();

    const int d = threadIdx.x;  // one head-dim element per thread
    for (int n = 0; n < ncols; ++n) {
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, sml[w * kDecodeCols + n].x);
      const float mu = mx == -INFINITY ? 0.f : mx;
      float acc = 0.f, sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float2 ml = sml[w * kDecodeCols + n];
        const float f = exp2f(ml.x - mu);
        acc += so[(w * kDecodeCols + n) * kColStride + d] * f;
        sum += ml.y * f;
      }
      if (nsplit == 1) {
        const int64_t t = qs + n / p.group;
        const int hq = h * p.group + n % p.group;
        const float v = empty_history ? 0.f : (sum > 0.f ? acc / sum : NAN);
        reinterpret_cast<T*>(p.out)[(t * p.num_q_heads + hq) * kDecodeHeadDim + d] =
            from_float<T>(v);
      } else {
        p.partial_o[((int64_t)item * kDecodeCols + n) * kDecodeHeadDim + d] = acc;
        if (d == 0) p.partial_ml[(int64_t)item * kDecodeCols + n] = make_float2(mx, sum);
      }
    }

    if (nsplit > 1) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        const int done = atomicAdd(p.merge_count + r * p.num_kv_heads + h, 1);
        s_last = done == nsplit - 1;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        for (int n = 0; n < ncols; ++n) {
          float mx = -INFINITY;
          for (int sp = 0; sp < nsplit; ++sp) {
            const int64_t it = (u0 + sp) * p.num_kv_heads + h;
            mx = fmaxf(mx, __ldcg(&p.partial_ml[it * kDecodeCols + n].x));
          }
          const float mu = mx == -INFINITY ? 0.f : mx;
          float acc = 0.f, sum = 0.f;
          for (int sp = 0; sp < nsplit; ++sp) {
            const int64_t it = (u0 + sp) * p.num_kv_heads + h;
            const float2 ml = __ldcg(&p.partial_ml[it * kDecodeCols + n]);
            const float f = exp2f(ml.x - mu);
            acc += __ldcg(&p.partial_o[(it * kDecodeCols + n) * kDecodeHeadDim + d]) * f;
            sum += ml.y * f;
          }
          const int64_t t = qs + n / p.group;
          const int hq = h * p.group + n % p.group;
          reinterpret_cast<T*>(p.out)[(t * p.num_q_heads + hq) * kDecodeHeadDim + d] =
              from_float<T>(sum > 0.f ? acc / sum : NAN);
        }
      }
    }
    __syncthreads();  // merge buffer and s_item are reused by the next item
  }
}

template <typename T, int STAGES>
int launch_typed(const DecodeParams& dp, cudaStream_t stream) {
  const int smem = STAGES * kWarps * kStageBytes;
  static_assert(kWarps * kDecodeCols * (kColStride + 2) * 4 <= STAGES * kWarps * kStageBytes,
                "merge buffer must fit in the ring");
  static int configured_device = -1;
  static int grid = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<T, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return MVB_ERR_CUDA;
    }
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_kernel<T, STAGES>,
                                                      kThreads, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return MVB_ERR_CUDA;
    }
    grid = num_sms() * (per_sm > 0 ? per_sm : 1);
    configured_device = dev;
  }
  paged_decode_kernel<T, STAGES><<<grid, kThreads, smem, stream>>>(dp);
  return check_launch();
}

}  // namespace

int launch_paged_decode(const AttentionProblem& a, const WorkspaceLayout& w) {
  char* ws = static_cast<char*>(a.workspace);
  DecodeParams dp;
  const int eb = 2;
  dp.query = static_cast<const char*>(a.query);
  dp.q_st_bytes = a.q_st * eb;
  dp.q_sh_bytes = a.q_sh * eb;
  dp.out = static_cast<char*>(a.out);
  dp.cache = static_cast<const char*>(a.cache);
  dp.plane_bytes = a.num_blocks * a.block_size * (int64_t)a.num_kv_heads * kRowBytes;
  dp.num_blocks = a.num_blocks;
  dp.block_size = a.block_size;
  dp.bs_shift = (a.block_size & (a.block_size - 1)) == 0 ? __builtin_ctz(a.block_size) : -1;
  dp.num_kv_heads = a.num_kv_heads;
  dp.group = a.num_q_heads / a.num_kv_heads;
  dp.num_q_heads = a.num_q_heads;
  dp.qpos = a.qpos;
  dp.qstart = a.qstart;
  dp.qsl = a.qsl;
  dp.ctx_len = a.ctx_len;
  dp.table = a.table;
  dp.table_stride = a.table_stride;
  dp.table_width = a.table_width;
  dp.num_requests = a.num_requests;
  dp.scale_log2 = a.scale * 1.4426950408889634f;
  dp.ctrl = reinterpret_cast<const int32_t*>(ws + w.ctrl);
  dp.cursor = reinterpret_cast<int32_t*>(ws + w.ctrl) + kCtrlCursor;
  dp.unit_prefix = reinterpret_cast<const int32_t*>(ws + w.unit_prefix);
  dp.merge_count = reinterpret_cast<int32_t*>(ws + w.merge_count);
  dp.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
  dp.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
  dp.status = a.status;
  if (a.dtype == MVB_DTYPE_F16) return launch_typed<__half, 3>(dp, a.stream);
  if (a.dtype == MVB_DTYPE_BF16) return launch_typed<__nv_bfloat16, 3>(dp, a.stream);
  return MVB_ERR_UNSUPPORTED_DTYPE;
}

}  // namespace mvb
