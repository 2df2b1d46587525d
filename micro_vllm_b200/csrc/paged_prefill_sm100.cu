// Varlen causal chunked-prefill attention over the paged cache on the
// 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128, fp16/bf16.
//
// Work item = (prefill-class request, 128-row query tile, KV head): the 128
// MMA rows are 128/G query tokens x the G query heads of one GQA group, so
// every K/V tile fetched serves the whole group.  A persistent grid (one
// CTA per SM, 224 KB of shared memory, 512 TMEM columns) pulls items from an
// atomic cursor, heaviest (latest) query tiles first.
//
// Roles inside a CTA (6 warps):
//   warp 0  TMA producer: the Q tile once per item (a 3-D tensor map over
//           [token, head, dim] so the G heads of a token land in adjacent
//           rows) and, per 128-key KV tile, the 8 pages of K and V (a 2-D
//           tensor map over the cache's [2*NB*bs slots, Hkv*128] view; one
//           16-row x 64-element box per page, plane and half) into a
//           2-stage ring, 128-byte swizzled — the layout the tensor cores
//           read directly.  Pages missing from the block table are fetched
//           from page 0 and masked.
//   warp 1  MMA issuer (one thread): S_j = Q.K_j^T into one of two TMEM
//           score buffers, then O += P_{j-1}.V_{j-1} with O resident in TMEM
//           (kind::f16, M=128, N=128, K=16 steps; V is read MN-major).
//   warps 2-5  softmax: one thread per row (= TMEM lane).  Each loads its
//           128 scores with tcgen05.ld, applies the causal / visibility
//           window mask, keeps an fp32 online softmax whose reference max
//           moves only when a new max exceeds it by 2^8 (then O is rescaled
//           in TMEM with tcgen05.ld/st — rare after the first tiles), writes
//           P in the swizzled K-major layout the PV MMA reads, zeroes V rows
//           no query may see (so stale cache bytes cannot reach O through
//           0 * NaN), and at the end normalises O and stores it.
// Every mbarrier wait is bounded; a timeout sets kStatusWaitTimeout and the
// kernel winds down.
//
// Semantics are those of ReferenceAttentionOperator.forward
// (reference.py:14-81), as in the decode kernel: token t of request r sees
// max(ctx_start[first token of r], ctx_start[t]) .. min(ctx_len[r]-1, pos[t]).
// Roofline: tensor cores; algorithmic flops per item = 4 * D * (visible
// query-key pairs) * heads.
#include <math.h>

#include <type_traits>

#include "mvb_common.cuh"
#include "mvb_internal.h"
#include "ptx_sm100.cuh"

namespace mvb {
namespace {

using namespace sm100;

constexpr int kRows = 128;                     // MMA M
constexpr int kKeys = 128;                     // keys per KV tile
constexpr int kHalf = kRows * 128;             // one [128 rows][64 elem] swizzled half: 16 KiB
constexpr int kTileBytes = 2 * kHalf;          // [128][128] fp16/bf16: 32 KiB
constexpr int kStageBytes = 2 * kTileBytes;    // K + V
constexpr int kStages = 2;
constexpr int kOffQ = 0;
constexpr int kOffKv = kTileBytes;
constexpr int kOffP = kOffKv + kStages * kStageBytes;
constexpr int kSmemUsed = kOffP + 2 * kTileBytes;  // Q + 2 KV stages + P (hi, lo) = 224 KiB
constexpr int kSmemBytes = kSmemUsed + 1024;       // + alignment slack
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;  // S buffers at columns 0 and 128, O at 256
constexpr float kRescaleLog2 = 8.f;

enum Bar : int {
  kQFull = 0,
  kKvFull = 1,    // +stage
  kKvEmpty = 3,   // +stage
  kSFull = 5,     // +buffer
  kSFree = 7,     // +buffer
  kPFull = 9,     // +buffer
  kPvDone = 11,   // +buffer
  kFinal = 13,    // last MMA commit before TMEM is released
  kNumBars = 14,
};

struct PrefillParams {
  char* out;
  int32_t num_q_heads, num_kv_heads, group, block_q, block_size, bs_shift;
  int64_t num_blocks, num_slots;
  const int64_t *qpos, *qstart, *qsl, *ctx_len, *table;
  int64_t table_stride, table_width;
  float scale_log2;
  const int64_t* ctrl;
  int32_t* cursor;
  const int64_t* unit_prefix;  // per request: first prefill unit (query tile)
  const int32_t* unit_req;     // unit -> request
  int32_t* status;
};

__device__ __forceinline__ int64_t page_of(const PrefillParams& p, const int64_t* trow,
                                           int64_t pos) {
  const int64_t lb = p.bs_shift >= 0 ? (pos >> p.bs_shift) : pos / p.block_size;
  if (pos < 0 || lb >= p.table_width) return -1;
  const int64_t blk = __ldg(trow + lb);
  return (blk >= 0 && blk < p.num_blocks) ? blk : -1;
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

struct Item {
  int64_t r, q0, q1, kbase, kv_lo, kv_hi;  // kv_[lo,hi] inclusive over the tile's rows
  int32_t h, n;                            // KV head, number of 128-key tiles
  bool empty_history;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kvmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int32_t item_sh;
  __shared__ unsigned long long kv_lo_sh, kv_hi_sh;
  __shared__ uint32_t page_ok_sh[kStages];
  __shared__ int32_t abort_sh;
  __shared__ int32_t last_issued[kStages];  // last KV tile index issued per stage
  __shared__ int32_t q_issued;              // Q loads issued (phase count of kQFull)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_items = p.ctrl[kCtrlPrefillUnits] * p.num_kv_heads;

  if (tid == 0) item_sh = atomicAdd(p.cursor, 1);
  __syncthreads();
  if (item_sh >= n_items) return;  // no prefill work for this CTA

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_addr(smem);
  const uint32_t bar0 = smem_addr(&bars[0]);
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };

  if (tid == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kKvFull + s), 1);
      mbar_init(bar(kKvEmpty + s), 1);
      mbar_init(bar(kSFull + s), 1);
      mbar_init(bar(kSFree + s), 4);
      mbar_init(bar(kPFull + s), 4);
      mbar_init(bar(kPvDone + s), 1);
    }
    mbar_init(bar(kFinal), 1);
    mbar_init_fence();
    abort_sh = 0;
    last_issued[0] = last_issued[1] = -1;
    q_issued = 0;
  }
  if (warp == 1) tmem_alloc(smem_addr(&tmem_base_sh), kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t idesc_qk = f16_idesc(kBf16, false, kRows, kKeys);
  const uint32_t idesc_pv = f16_idesc(kBf16, true, kRows, 128);

  uint32_t kvc = 0;       // KV tiles consumed so far by this CTA (ring / buffer phases)
  uint32_t item_cnt = 0;  // items processed (Q barrier phase)

  for (;;) {
    const int64_t claimed = item_sh;
    if (claimed >= n_items) break;
    // ---- describe the item (heaviest query tiles first) ----
    const int64_t it = n_items - 1 - claimed;
    Item I;
    I.h = (int32_t)(it % p.num_kv_heads);
    const int64_t unit = it / p.num_kv_heads;
    I.r = __ldg(p.unit_req + unit);
    const int64_t qt = unit - __ldg(p.unit_prefix + I.r);
    const int64_t qs = __ldg(p.qsl + I.r), qe = __ldg(p.qsl + I.r + 1);
    I.q0 = qs + qt * p.block_q;
    I.q1 = min(I.q0 + (int64_t)p.block_q, qe);
    const int64_t gather_lo = max(__ldg(p.qstart + qs), (int64_t)0);
    const int64_t clen = __ldg(p.ctx_len + I.r);
    I.empty_history = clen <= gather_lo;

    // Per-row visibility window (softmax threads own rows).
    const int row = 32 * (warp & 3) + lane;
    const int64_t tok = I.q0 + row / p.group;
    const bool row_valid = warp >= 2 && tok < I.q1;
    int64_t lo_q = 1, hi_q = 0;
    if (row_valid) {
      lo_q = max(gather_lo, __ldg(p.qstart + tok));
      hi_q = min(clen - 1, __ldg(p.qpos + tok));
    }
    if (tid == 0) {
      kv_lo_sh = ~0ull;
      kv_hi_sh = 0ull;
    }
    __syncthreads();
    if (row_valid && lo_q <= hi_q) {
      atomicMin(&kv_lo_sh, (unsigned long long)lo_q);
      atomicMax(&kv_hi_sh, (unsigned long long)(hi_q + 1));
    }
    __syncthreads();
    const bool any = kv_hi_sh > 0ull && kv_lo_sh != ~0ull;
    I.kv_lo = any ? (int64_t)kv_lo_sh : 0;
    I.kv_hi = any ? (int64_t)kv_hi_sh - 1 : -1;
    I.kbase = I.kv_lo & ~(int64_t)15;
    I.n = any ? (int32_t)((I.kv_hi - I.kbase) / kKeys + 1) : 0;
    const int64_t* trow = p.table + I.r * p.table_stride;

    if (I.n > 0) {
      if (warp == 0) {
        // ------------------------------------------------ producer
        if (lane == 0) {
          mbar_expect_tx(bar(kQFull), kTileBytes);
          const int32_t qy = I.h * p.group, qz = (int32_t)I.q0;
          tma_load_3d(sb + kOffQ, &qmap, 0, qy, qz, bar(kQFull));
          tma_load_3d(sb + kOffQ + kHalf, &qmap, 64, qy, qz, bar(kQFull));
          q_issued = (int32_t)item_cnt + 1;
        }
        for (int j = 0; j < I.n; ++j) {
          const uint32_t c = kvc + j, s = c & 1, ph = (c >> 1) & 1;
          if (!mbar_wait(bar(kKvEmpty + s), ph ^ 1)) {
            if (lane == 0) atomicOr(&abort_sh, 1);
            break;
          }
          const int64_t pos = I.kbase + (int64_t)j * kKeys + 16 * lane;
          int64_t blk = -1;
          if (lane < 8) blk = page_of(p, trow, pos);
          const bool ok = blk >= 0;
          const uint32_t mask = __ballot_sync(0xffffffffu, ok) & 0xffu;
          if (lane == 0) {
            page_ok_sh[s] = mask;
            mbar_expect_tx(bar(kKvFull + s), kStageBytes);
          }
          __syncwarp();
          if (lane == 0) last_issued[s] = (int32_t)c;
          if (lane < 8) {
            const int64_t page = ok ? blk : 0;
            const int64_t off = p.bs_shift >= 0 ? (pos & (p.block_size - 1)) : pos % p.block_size;
            const int32_t y = (int32_t)(page * p.block_size + off);
            const int32_t x = I.h * 128;
            const uint32_t k_dst = sb + kOffKv + s * kStageBytes + lane * 2048;
            const uint32_t v_dst = k_dst + kTileBytes;
            tma_load_2d(k_dst, &kvmap, x, y, bar(kKvFull + s));
            tma_load_2d(k_dst + kHalf, &kvmap, x + 64, y, bar(kKvFull + s));
            tma_load_2d(v_dst, &kvmap, x, y + (int32_t)p.num_slots, bar(kKvFull + s));
            tma_load_2d(v_dst + kHalf, &kvmap, x + 64, y + (int32_t)p.num_slots, bar(kKvFull + s));
          }
        }
      } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
          bool ok = mbar_wait(bar(kQFull), item_cnt & 1);
          tc_fence_after();
          for (int j = 0; ok && j <= I.n; ++j) {
            if (j < I.n) {
              const uint32_t c = kvc + j, s = c & 1, ph = (c >> 1) & 1;
              ok = mbar_wait(bar(kKvFull + s), ph) && mbar_wait(bar(kSFree + s), ph ^ 1);
              if (!ok) break;
              tc_fence_after();
              const uint32_t kb = sb + kOffKv + s * kStageBytes;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
                umma_f16(tmem + s * kKeys, sw128_desc(sb + kOffQ + off, 16, 1024),
                         sw128_desc(kb + off, 16, 1024), idesc_qk, k > 0);
              }
              umma_commit(bar(kSFull + s));
            }
            if (j >= 1) {
              const uint32_t c = kvc + j - 1, s = c & 1, ph = (c >> 1) & 1;
              ok = mbar_wait(bar(kPFull + s), ph);
              if (!ok) break;
              tc_fence_after();
              const uint32_t vb = sb + kOffKv + s * kStageBytes + kTileBytes;
#pragma unroll
              for (int part = 0; part < (kBf16 ? 2 : 1); ++part) {  // P_hi (+ P_lo in bf16)
                const uint32_t pb = sb + kOffP + part * kTileBytes;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  umma_f16(tmem + kTmemO,
                           sw128_desc(pb + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024),
                           sw128_desc(vb + k * 2048, kHalf, 1024), idesc_pv,
                           (j > 1) || (k > 0) || (part > 0));
                }
              }
              umma_commit(bar(kKvEmpty + s));
              umma_commit(bar(kPvDone + s));
            }
          }
          if (!ok) atomicOr(&abort_sh, 1);
        }
        __syncwarp();
      } else {
        // ------------------------------------------------ softmax / epilogue
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < I.n; ++j) {
          const uint32_t c = kvc + j, s = c & 1, ph = (c >> 1) & 1;
          ok = mbar_wait(bar(kSFull + s), ph) && mbar_wait(bar(kKvFull + s), ph);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          float sv[kKeys];
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            float tmp[32];
            tmem_ld32(tmem + lane_base + s * kKeys + 32 * ch, tmp);
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[32 * ch + i] = tmp[i];
          }
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kSFree + s));

          const int64_t k0 = I.kbase + (int64_t)j * kKeys;
          const uint32_t pok = page_ok_sh[s];
          const bool whole = row_valid && k0 >= lo_q && k0 + kKeys - 1 <= hi_q && pok == 0xffu;
          float tmax = -INFINITY;
          if (whole) {
#pragma unroll
            for (int i = 0; i < kKeys; ++i) {
              sv[i] *= p.scale_log2;
              tmax = fmaxf(tmax, sv[i]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < kKeys; ++i) {
              const int64_t key = k0 + i;
              const bool vis = row_valid && key >= lo_q && key <= hi_q && ((pok >> (i >> 4)) & 1u);
              sv[i] = vis ? sv[i] * p.scale_log2 : -INFINITY;
              tmax = fmaxf(tmax, sv[i]);
            }
          }
          float corr = 1.f;
          if (tmax > m_ref + kRescaleLog2) {
            corr = exp2f(m_ref - tmax);  // 0 when m_ref is -inf
            l *= corr;
            m_ref = tmax;
          }
          // PV_{j-1} done: O may be rescaled and the P buffer it read is free.
          if (j >= 1) {
            const uint32_t cp = c - 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(kPvDone + (cp & 1)), (cp >> 1) & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
              for (int ch = 0; ch < 4; ++ch) {
                float o[32];
                tmem_ld32(tmem + lane_base + kTmemO + 32 * ch, o);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] *= corr;
                tmem_st32(tmem + lane_base + kTmemO + 32 * ch, o);
              }
              tmem_wait_st();
            }
          }
          const float mu = m_ref == -INFINITY ? 0.f : m_ref;
          float psum = 0.f;
          // P goes to the A operand of the P.V MMA.  In bf16 (8-bit mantissa)
          // it is split into P_hi + P_lo, both bf16, so P keeps ~16 bits and
          // the two MMAs into O match the fp16 path's accuracy.
          uint8_t* prow = smem + kOffP + row * 128;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              uint32_t w[4], wl[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = half * 64 + cc * 8 + 2 * e;
                const float a = exp2f(sv[i] - mu), b = exp2f(sv[i + 1] - mu);
                psum += a + b;
                w[e] = pack2<T>(a, b);
                if constexpr (kBf16) {
                  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
                  const float2 hf = __bfloat1622float2(hi);
                  wl[e] = pack2<T>(a - hf.x, b - hf.y);
                }
              }
              const int off = half * kHalf + ((cc ^ (row & 7)) << 4);
              *reinterpret_cast<uint4*>(prow + off) = make_uint4(w[0], w[1], w[2], w[3]);
              if constexpr (kBf16)
                *reinterpret_cast<uint4*>(prow + kTileBytes + off) =
                    make_uint4(wl[0], wl[1], wl[2], wl[3]);
            }
          }
          l += psum;
          // Zero V rows no query of this tile may see (below the window,
          // past the last query, or on a missing page): they hold stale or
          // sentinel bytes that must not reach O as 0 * NaN.
          {
            const int64_t key = k0 + row;
            if (key < I.kv_lo || key > I.kv_hi || !((pok >> (row >> 4)) & 1u)) {
              uint8_t* vrow = smem + kOffKv + s * kStageBytes + kTileBytes + row * 128;
              const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
              for (int cc = 0; cc < 8; ++cc) {
                *reinterpret_cast<uint4*>(vrow + cc * 16) = z;
                *reinterpret_cast<uint4*>(vrow + kHalf + cc * 16) = z;
              }
            }
          }
          fence_proxy_async();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kPFull + s));
        }
        // ---- epilogue: O / l -> output rows ----
        const uint32_t cl = kvc + I.n - 1;
        if (ok && __all_sync(0xffffffffu, mbar_wait(bar(kPvDone + (cl & 1)), (cl >> 1) & 1))) {
          tc_fence_after();
          const float inv = l > 0.f ? 1.f / l : NAN;
          T* orow = reinterpret_cast<T*>(p.out) +
                    (tok * p.num_q_heads + I.h * p.group + row % p.group) * 128;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            float o[32];
            tmem_ld32(tmem + lane_base + kTmemO + 32 * ch, o);
            tmem_wait_ld();
            if (row_valid) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 q;
                q.x = pack2<T>(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
                q.y = pack2<T>(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
                q.z = pack2<T>(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
                q.w = pack2<T>(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
                *reinterpret_cast<uint4*>(orow + 32 * ch + 8 * v) = q;
              }
            }
          }
          tc_fence_before();
        } else {
          ok = false;
        }
        if (!ok && lane == 0) atomicOr(&abort_sh, 1);
      }
    } else if (warp >= 2 && row_valid) {
      // No visible key at all: 0 for an empty gathered history, else NaN
      // (softmax over an all -inf row), as the reference.
      const float v = I.empty_history ? 0.f : NAN;
      T* orow = reinterpret_cast<T*>(p.out) +
                (tok * p.num_q_heads + I.h * p.group + row % p.group) * 128;
      const uint32_t pv = pack2<T>(v, v);
      for (int i = 0; i < 16; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(pv, pv, pv, pv);
    }

    kvc += (uint32_t)I.n;
    if (I.n > 0) ++item_cnt;  // kQFull completes one phase per item with work
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (abort_sh) {
      if (tid == 0 && p.status != nullptr) atomicOr(p.status, kStatusWaitTimeout);
      break;
    }
    if (tid == 0) item_sh = atomicAdd(p.cursor, 1);
    __syncthreads();
  }

  // Everything this CTA issued lands before TMEM and shared memory go away
  // (each wait bounded): the MMA thread waits on a final commit; after an
  // abort, thread 0 also waits for the last TMA loads of each buffer.
  if (warp == 1 && lane == 0) {
    umma_commit(bar(kFinal));
    mbar_wait(bar(kFinal), 0);
  }
  if (tid == 0 && abort_sh) {
    for (int s = 0; s < kStages; ++s)
      if (last_issued[s] >= 0) mbar_wait(bar(kKvFull + s), (last_issued[s] >> 1) & 1);
    if (q_issued > 0) mbar_wait(bar(kQFull), (q_issued - 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------ host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  }
  return fn;
}

}  // namespace

bool prefill_tc_supported(const AttentionProblem& a) {
  const int group = a.num_q_heads / a.num_kv_heads;
  const int64_t num_slots = a.num_blocks * a.block_size;
  return (a.dtype == MVB_DTYPE_F16 || a.dtype == MVB_DTYPE_BF16) && a.head_dim == 128 &&
         group >= 1 && group <= 16 && (kRows % group) == 0 && (a.block_size % 16) == 0 &&
         ((uintptr_t)a.query % 16) == 0 && ((uintptr_t)a.cache % 16) == 0 &&
         ((uintptr_t)a.out % 16) == 0 && (a.q_st % 8) == 0 && (a.q_sh % 8) == 0 &&
         a.q_sh >= 128 && 2 * num_slots < ((int64_t)1 << 31) && a.num_tokens < ((int64_t)1 << 31) &&
         encoder() != nullptr;
}

int launch_paged_prefill(const AttentionProblem& a, const WorkspaceLayout& w) {
  EncodeTiled encode = encoder();
  if (encode == nullptr) return MVB_ERR_CUDA;
  const CUtensorMapDataType dt =
      a.dtype == MVB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int group = a.num_q_heads / a.num_kv_heads;
  const int64_t num_slots = a.num_blocks * a.block_size;

  CUtensorMap qmap, kvmap;
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)a.num_q_heads, (cuuint64_t)a.num_tokens};
    const cuuint64_t strides[2] = {(cuuint64_t)a.q_sh * 2, (cuuint64_t)a.q_st * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(kRows / group)};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&qmap, dt, 3, const_cast<void*>(a.query), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return MVB_ERR_UNSUPPORTED_SHAPE;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.num_kv_heads * 128, (cuuint64_t)(2 * num_slots)};
    const cuuint64_t strides[1] = {(cuuint64_t)a.num_kv_heads * 128 * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&kvmap, dt, 2, const_cast<void*>(a.cache), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return MVB_ERR_UNSUPPORTED_SHAPE;
  }

  char* ws = static_cast<char*>(a.workspace);
  PrefillParams pp;
  pp.out = static_cast<char*>(a.out);
  pp.num_q_heads = a.num_q_heads;
  pp.num_kv_heads = a.num_kv_heads;
  pp.group = group;
  pp.block_q = kRows / group;
  pp.block_size = a.block_size;
  pp.bs_shift = (a.block_size & (a.block_size - 1)) == 0 ? __builtin_ctz(a.block_size) : -1;
  pp.num_blocks = a.num_blocks;
  pp.num_slots = num_slots;
  pp.qpos = a.qpos;
  pp.qstart = a.qstart;
  pp.qsl = a.qsl;
  pp.ctx_len = a.ctx_len;
  pp.table = a.table;
  pp.table_stride = a.table_stride;
  pp.table_width = a.table_width;
  pp.scale_log2 = a.scale * 1.4426950408889634f;
  pp.ctrl = reinterpret_cast<const int64_t*>(ws + w.ctrl);
  pp.cursor = reinterpret_cast<int32_t*>(reinterpret_cast<int64_t*>(ws + w.ctrl) + kCtrlPrefillCursor);
  pp.unit_prefix = reinterpret_cast<const int64_t*>(ws + w.prefill_prefix);
  pp.unit_req = reinterpret_cast<const int32_t*>(ws + w.prefill_unit_req);
  pp.status = a.status;

  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(paged_prefill_kernel<__half>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_prefill_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return MVB_ERR_CUDA;
    }
    configured_device = dev;
  }
  const int grid = num_sms();
  if (a.dtype == MVB_DTYPE_BF16)
    paged_prefill_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, a.stream>>>(qmap, kvmap, pp);
  else
    paged_prefill_kernel<__half><<<grid, kThreads, kSmemBytes, a.stream>>>(qmap, kvmap, pp);
  return check_launch();
}

}  // namespace mvb
