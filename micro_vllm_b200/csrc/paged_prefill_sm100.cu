// Varlen causal chunked-prefill attention over the paged cache on the
// 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128, fp16/bf16.
//
// Work item = (prefill-class request, pair of 128-row query tiles, KV head).
// Each tile's 128 MMA rows are 128/G query tokens x the G query heads of one
// GQA group; the two tiles (A: the earlier tokens, B: the next ones) share
// every K/V tile fetched.  A persistent grid (one CTA per SM, 225 KB of
// shared memory, all 512 TMEM columns) pulls items from an atomic cursor,
// heaviest (latest) query tiles first.
//
// Roles inside a CTA (11 warps):
//   warps 0, 10  TMA producers (K with Q, and V): both Q tiles once per item (a 3-D tensor map over
//           [token, head, dim] so the G heads of a token land in adjacent
//           rows) and, per 128-key KV tile, the 8 pages of K and V (a 2-D
//           tensor map over the cache's [2*NB*bs slots, Hkv*128] view; one
//           16-row x 64-element box per page, plane and half) into a
//           2-stage K ring and a 3-stage V ring, 128-byte swizzled — the layout the tensor cores
//           read directly.  Pages missing from the block table are fetched
//           from page 0 and masked.
//   warp 1  MMA issuer (one thread), ping-pong between the tiles:
//             S_A(0), S_B(0); then per KV tile j:
//             PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)
//           S_X = Q_X.K^T lands in TMEM (128 fp32 columns per tile); the
//           softmax writes P_X back over S_X as packed 16-bit pairs and
//           PV_X: O_X += P_X.V_j reads it straight from TMEM (A operand in
//           TMEM, V from shared memory MN-major).  tcgen05 operations of one
//           thread complete in issue order, so S_X(j+1) finishing implies
//           PV_X(j) finished.
//   warps 2-5 / 6-9  softmax of tile A / B, one thread per row (= TMEM
//           lane): pass 1 loads the 128 scores and takes the masked max;
//           the reference max moves only when the tile max exceeds it by
//           2^8, and then O_X is rescaled in TMEM (no wait needed: O_X holds
//           PV_X(j-1), complete since S_X(j) is); pass 2 reloads the scores,
//           computes P = 2^(s - max) and stores it to TMEM.  bf16 P is split
//           into P_hi + P_lo (two MMAs) to keep ~16 bits.  Tile A's warps
//           also zero V rows no query of the pair may see, so stale cache
//           bytes cannot reach O as 0 * NaN.  At the end each row's O is
//           normalised and stored.
// Every mbarrier wait is bounded; a timeout sets kStatusWaitTimeout and the
// kernel winds down.
//
// Semantics are those of ReferenceAttentionOperator.forward
// (reference.py:14-81), as in the decode kernel: token t of request r sees
// max(ctx_start[first token of r], ctx_start[t]) .. min(ctx_len[r]-1, pos[t]).
// Roofline: tensor cores; algorithmic flops per request = 4 * D * Hq *
// (visible query-key pairs).
#include <math.h>

#include <type_traits>

#include "mvb_common.cuh"
#include "mvb_internal.h"
#include "ptx_sm100.cuh"

namespace mvb {
namespace {

using namespace sm100;

constexpr int kRows = 128;                   // MMA M: rows of one query tile
constexpr int kKeys = 128;                   // keys per KV tile
constexpr int kHalf = kRows * 128;           // [128 rows][64 elem] swizzled half: 16 KiB
constexpr int kTileBytes = 2 * kHalf;        // [128][128] 16-bit: 32 KiB
constexpr int kKStages = 2;                  // K ring (released right after the S MMAs)
constexpr int kVStages = 3;                  // V ring (released after the P.V MMAs)
constexpr int kOffQ = 0;                     // Q_A, Q_B
constexpr int kOffK = 2 * kTileBytes;
constexpr int kOffV = kOffK + kKStages * kTileBytes;
constexpr int kSmemUsed = kOffV + kVStages * kTileBytes;  // 224 KiB
constexpr int kSmemBytes = kSmemUsed + 1024;               // + alignment slack
constexpr int kThreads = 352;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S/P of tile A and B, then O of tile A and B.
__device__ __forceinline__ uint32_t col_s(int t) { return 128u * (uint32_t)t; }
__device__ __forceinline__ uint32_t col_o(int t) { return 256u + 128u * (uint32_t)t; }
constexpr float kRescaleLog2 = 8.f;

// mbarrier indices, derived from the ring depths so no two overlap.
enum Bar : int {
  kQFull = 0,
  kKFull = kQFull + 1,           // +K slot: K tile landed
  kKEmpty = kKFull + kKStages,   // +K slot: every S MMA read it
  kVFull = kKEmpty + kKStages,   // +V slot: V tile landed
  kVEmpty = kVFull + kVStages,   // +V slot: every P.V MMA read it
  kSFull = kVEmpty + kVStages,   // +tile (A, B)
  kPFull = kSFull + 2,           // +tile
  kPvDone = kPFull + 2,          // +tile
  kFinal = kPvDone + 2,          // last MMA commit before TMEM is released
  kNumBars = kFinal + 1,
};
static_assert(kNumBars == 1 + 2 * kKStages + 2 * kVStages + 3 * 2 + 1, "mbarrier layout");

// Ring slot and phase of the c-th KV tile this CTA processes.
__device__ __forceinline__ uint32_t kslot(uint32_t c) { return c % kKStages; }
__device__ __forceinline__ uint32_t kphase(uint32_t c) { return (c / kKStages) & 1; }
__device__ __forceinline__ uint32_t vslot(uint32_t c) { return c % kVStages; }
__device__ __forceinline__ uint32_t vphase(uint32_t c) { return (c / kVStages) & 1; }

struct PrefillParams {
  char* out;
  int32_t num_q_heads, num_kv_heads, group, block_q, block_size, bs_shift;
  int64_t num_blocks, num_slots;
  const int64_t *qpos, *qstart, *qsl, *ctx_len, *table;
  int64_t table_stride, table_width;
  float scale_log2;
  const int64_t* ctrl;
  int32_t* cursor;
  const int64_t* unit_prefix;  // per request: first prefill unit (query-tile pair)
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

// 11 warps: the busiest SM sub-partition holds 3 of them, so a thread may
// use at most 168 registers (16 K registers per sub-partition).
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kvmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int32_t item_sh;
  __shared__ unsigned long long kv_lo_sh, kv_hi_sh;
  __shared__ int32_t abort_sh;
  __shared__ int32_t last_issued[2];  // last K and last V tile index issued
  __shared__ int32_t q_issued;              // Q loads issued (phases of kQFull)

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
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
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar(kKFull + s), 1);
      mbar_init(bar(kKEmpty + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(bar(kVFull + s), 1);
      mbar_init(bar(kVEmpty + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kSFull + s), 1);
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

  const uint32_t idesc_qk = f16_idesc(kBf16, false, kRows, kKeys);
  const uint32_t idesc_pv = f16_idesc(kBf16, true, kRows, 128);

  // Running counts (identical in every role): KV tiles of this CTA (ring
  // phases), tiles processed per query tile (S/P/PV phases), Q loads.
  uint32_t kvc = 0, tc0 = 0, tc1 = 0, qc = 0;
  // Softmax role of this warp: tile 0 (A) for warps 2-5, 1 (B) for 6-9.
  const int x = warp >= 6 ? 1 : 0;
  const int row = 32 * (warp & 3) + lane;  // TMEM lane of this thread

  for (;;) {
    const int64_t claimed = item_sh;
    if (claimed >= n_items) break;
    // ---- describe the item (heaviest query tiles first) ----
    const int64_t it = n_items - 1 - claimed;
    const int h = (int)(it % p.num_kv_heads);
    const int64_t unit = it / p.num_kv_heads;
    const int64_t r = __ldg(p.unit_req + unit);
    const int64_t qt = unit - __ldg(p.unit_prefix + r);
    const int64_t qs = __ldg(p.qsl + r), qe = __ldg(p.qsl + r + 1);
    const int64_t q0 = qs + qt * 2 * p.block_q;  // first token of tile A
    const bool b_active = q0 + p.block_q < qe;
    const int64_t gather_lo = max(__ldg(p.qstart + qs), (int64_t)0);
    const int64_t clen = __ldg(p.ctx_len + r);
    const bool empty_history = clen <= gather_lo;

    // Per-row visibility window (softmax threads own rows).  Positions fit
    // 32 bits: the planner refuses contexts longer than 2^30.
    const int64_t tok = q0 + (int64_t)x * p.block_q + row / p.group;
    const bool row_valid =
        warp >= 2 && warp < 10 && tok < min(qe, q0 + (int64_t)(x + 1) * p.block_q);
    int32_t lo_q = 1, hi_q = 0;
    if (row_valid) {
      lo_q = (int32_t)min(max(gather_lo, __ldg(p.qstart + tok)), kMaxContext);
      hi_q = (int32_t)max(min(clen - 1, __ldg(p.qpos + tok)), (int64_t)-1);
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
    const int32_t kv_lo = any ? (int32_t)kv_lo_sh : 0;
    const int32_t kv_hi = any ? (int32_t)kv_hi_sh - 1 : -1;
    const int32_t kbase = kv_lo & ~15;
    const int n = any ? (kv_hi - kbase) / kKeys + 1 : 0;
    const int64_t* trow = p.table + r * p.table_stride;
    const int ntiles = b_active ? 2 : 1;

    if (n > 0) {
      if (warp == 0 || warp == 10) {
        // ------------------------------------------------ producers
        // Warp 0 loads Q and the K tiles, warp 10 the V tiles; each waits
        // only on its own ring, so K is never held up behind a V slot.
        const bool is_k = warp == 0;
        if (is_k && lane == 0) {
          mbar_expect_tx(bar(kQFull), ntiles * kTileBytes);
          for (int t = 0; t < ntiles; ++t) {
            const int32_t qy = h * p.group, qz = (int32_t)(q0 + (int64_t)t * p.block_q);
            tma_load_3d(sb + kOffQ + t * kTileBytes, &qmap, 0, qy, qz, bar(kQFull));
            tma_load_3d(sb + kOffQ + t * kTileBytes + kHalf, &qmap, 64, qy, qz, bar(kQFull));
          }
          q_issued = (int32_t)qc + 1;
        }
        for (int j = 0; j < n; ++j) {
          const uint32_t c = kvc + j;
          const uint32_t slot = is_k ? kslot(c) : vslot(c);
          const uint32_t full = bar((is_k ? kKFull : kVFull) + slot);
          // K(j) reuses the slot of K(j-2), free once every S(j-2) MMA ran;
          // V(j) that of V(j-3), free once every P.V(j-3) MMA ran.
          const uint32_t empty_phase = (is_k ? kphase(c) : vphase(c)) ^ 1;
          if (!mbar_wait(bar((is_k ? kKEmpty : kVEmpty) + slot), empty_phase)) {
            if (lane == 0) atomicOr(&abort_sh, 1);
            break;
          }
          const int64_t pos = (int64_t)kbase + (int64_t)j * kKeys + 16 * lane;
          int64_t blk = -1;
          if (lane < 8) blk = page_of(p, trow, pos);
          if (lane == 0) {
            last_issued[is_k ? 0 : 1] = (int32_t)c;
            mbar_expect_tx(full, kTileBytes);
          }
          __syncwarp();
          if (lane < 8) {
            // Missing pages load page 0; the softmax masks their keys.
            const int64_t page = blk >= 0 ? blk : 0;
            const int64_t off = p.bs_shift >= 0 ? (pos & (p.block_size - 1)) : pos % p.block_size;
            const int32_t y = (int32_t)(page * p.block_size + off) + (is_k ? 0 : (int32_t)p.num_slots);
            const int32_t xk = h * 128;
            const uint32_t dst = sb + (is_k ? kOffK : kOffV) + slot * kTileBytes + lane * 2048;
            tma_load_2d(dst, &kvmap, xk, y, full);
            tma_load_2d(dst + kHalf, &kvmap, xk + 64, y, full);
          }
        }
      } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
          auto issue_s = [&](int t, uint32_t stage) {
            const uint32_t kb = sb + kOffK + stage * kTileBytes;
            const uint32_t qb = sb + kOffQ + t * kTileBytes;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
              umma_f16(tmem + col_s(t), sw128_desc(qb + off, 16, 1024),
                       sw128_desc(kb + off, 16, 1024), idesc_qk, k > 0);
            }
            umma_commit(bar(kSFull + t));
          };
          auto issue_pv = [&](int t, uint32_t stage, bool acc) {
            const uint32_t vb = sb + kOffV + stage * kTileBytes;
#pragma unroll
            for (int part = 0; part < (kBf16 ? 2 : 1); ++part) {  // P_hi (+ P_lo in bf16)
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const uint32_t pcol = col_s(t) + 32 * (k >> 1) + 8 * (k & 1) + 16 * part;
                umma_f16_ts(tmem + col_o(t), tmem + pcol, sw128_desc(vb + k * 2048, kHalf, 1024),
                            idesc_pv, acc || k > 0 || part > 0);
              }
            }
            umma_commit(bar(kPvDone + t));
          };
          bool ok = mbar_wait(bar(kQFull), qc & 1) &&
                    mbar_wait(bar(kKFull + kslot(kvc)), kphase(kvc));
          if (ok) {
            tc_fence_after();
            for (int t = 0; t < ntiles; ++t) issue_s(t, kslot(kvc));
            umma_commit(bar(kKEmpty + kslot(kvc)));  // K(0) read by every S(0)
          }
          for (int j = 0; ok && j < n; ++j) {
            const uint32_t c = kvc + j, sv = vslot(c);
            const uint32_t cn = c + 1, skn = kslot(cn);
            for (int t = 0; t < ntiles; ++t) {
              ok = mbar_wait(bar(kPFull + t), ((t == 0 ? tc0 : tc1) + j) & 1);
              if (ok && t == 0) ok = mbar_wait(bar(kVFull + sv), vphase(c));
              if (!ok) break;
              tc_fence_after();
              issue_pv(t, sv, j > 0);
              if (t == ntiles - 1) umma_commit(bar(kVEmpty + sv));  // V(j) read by every P.V(j)
              if (j + 1 < n) {
                if (t == 0) {
                  ok = mbar_wait(bar(kKFull + skn), kphase(cn));
                  if (!ok) break;
                  tc_fence_after();
                }
                issue_s(t, skn);
                if (t == ntiles - 1) umma_commit(bar(kKEmpty + skn));  // K(j+1) read by every S
              }
            }
          }
          if (!ok) atomicOr(&abort_sh, 1);
        }
        __syncwarp();
      } else if (x == 0 || b_active) {
        // ------------------------------------------------ softmax / epilogue of tile x
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t s_cols = tmem + lane_base + col_s(x);
        const uint32_t o_cols = tmem + lane_base + col_o(x);
        const uint32_t tcx = x == 0 ? tc0 : tc1;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
          const uint32_t c = kvc + j, sv = vslot(c);
          const int32_t k0 = kbase + j * kKeys;
          // Pages of this KV tile that exist in the block table (lanes 0-7
          // look up one 16-key page each; loaded before the wait).
          uint32_t pok;
          {
            int64_t blk = -1;
            if (lane < 8) blk = page_of(p, trow, (int64_t)k0 + 16 * lane);
            pok = __ballot_sync(0xffffffffu, blk >= 0) & 0xffu;
          }
          ok = mbar_wait(bar(kSFull + x), (tcx + j) & 1);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // All 128 scores of this row in one batch of TMEM loads.
          uint32_t sc[4][32];
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tmem_ld32_raw(s_cols + 32 * ch, sc[ch]);
          tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) reg_fence(sc[ch]);
          // Visible keys of this row inside the tile: [lo_rel, hi_rel) on
          // valid pages.  Hidden scores become -inf once, here.
          int lo_rel = 0, hi_rel = 0;
          if (row_valid) {
            lo_rel = min(max(lo_q - k0, 0), kKeys);
            hi_rel = min(max(hi_q - k0 + 1, 0), kKeys);
          }
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          if (lo_rel == 0 && hi_rel == kKeys && pok == 0xffu) {
#pragma unroll
            for (int i = 0; i < kKeys; ++i)
              mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(sc[i >> 5][i & 31]));
          } else {
#pragma unroll
            for (int i = 0; i < kKeys; ++i) {
              const bool vis = i >= lo_rel && i < hi_rel && ((pok >> (i >> 4)) & 1u);
              const float v = vis ? __uint_as_float(sc[i >> 5][i & 31]) : -INFINITY;
              sc[i >> 5][i & 31] = __float_as_uint(v);
              mx[i & 3] = fmaxf(mx[i & 3], v);
            }
          }
          // scale > 0, so the max of the scaled scores is the scaled max.
          const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.scale_log2;
          float corr = 1.f;
          if (tmax > m_ref + kRescaleLog2) {
            corr = ex2(m_ref - tmax);  // 0 when m_ref is -inf
            l *= corr;
            m_ref = tmax;
          }
          // O holds PV(j-1), complete because S(j) (issued after it) is.
          if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
            for (int ch = 0; ch < 8; ++ch) {  // 16 columns at a time: the scores stay live
              uint32_t o[16];
              tmem_ld16_raw(o_cols + 16 * ch, o);
              tmem_wait_ld();
              reg_fence(o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
              tmem_st16(o_cols + 16 * ch, o);
            }
          }
          // P = 2^(s*scale - m_ref), written over S as packed 16-bit pairs:
          // keys 32ch..32ch+31 -> columns 32ch..32ch+15 (P_hi) and
          // 32ch+16..32ch+31 (P_lo, bf16 only), behind the scores already read.
          const float mu = m_ref == -INFINITY ? 0.f : m_ref;
          float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {  // 16 keys: 8 packed columns per store
              uint32_t hi[8], lo[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int i = 16 * hh + 2 * e;
                const float pa = ex2(fmaf(__uint_as_float(sc[ch][i]), p.scale_log2, -mu));
                const float pb = ex2(fmaf(__uint_as_float(sc[ch][i + 1]), p.scale_log2, -mu));
                ps[e & 3] += pa + pb;
                hi[e] = pack2<T>(pa, pb);
                if constexpr (kBf16) {
                  const float2 hf =
                      __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hi[e]));
                  lo[e] = pack2<T>(pa - hf.x, pb - hf.y);
                }
              }
              tmem_st8(s_cols + 32 * ch + 8 * hh, hi);
              if constexpr (kBf16) tmem_st8(s_cols + 32 * ch + 16 + 8 * hh, lo);
            }
          }
          tmem_wait_st();
          const float psum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
          l += psum;
          if (x == 0) {
            // Zero V rows no query of the pair may see (below the window,
            // past the last query, or on a missing page): they hold stale or
            // sentinel bytes that must not reach O as 0 * NaN.
            const int32_t key = k0 + row;
            if (key < kv_lo || key > kv_hi || !((pok >> (row >> 4)) & 1u)) {
              // V(j) must have landed before its rows are overwritten.
              if (!mbar_wait(bar(kVFull + sv), vphase(c))) atomicOr(&abort_sh, 1);
              uint8_t* vrow = smem + kOffV + sv * kTileBytes + row * 128;
              const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
              for (int cc = 0; cc < 8; ++cc) {
                *reinterpret_cast<uint4*>(vrow + cc * 16) = z;
                *reinterpret_cast<uint4*>(vrow + kHalf + cc * 16) = z;
              }
            }
            fence_proxy_async();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kPFull + x));
        }
        // ---- epilogue: O / l -> output rows ----
        if (ok && __all_sync(0xffffffffu, mbar_wait(bar(kPvDone + x), (tcx + n - 1) & 1))) {
          tc_fence_after();
          const float inv = l > 0.f ? 1.f / l : NAN;
          T* orow = reinterpret_cast<T*>(p.out) +
                    (tok * p.num_q_heads + h * p.group + row % p.group) * 128;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            float o[32];
            tmem_ld32(o_cols + 32 * ch, o);
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
        } else {
          ok = false;
        }
        if (!ok && lane == 0) atomicOr(&abort_sh, 1);
      }
    } else if (warp >= 2 && row_valid) {
      // No visible key at all: 0 for an empty gathered history, else NaN
      // (softmax over an all -inf row), as the reference.
      const float v = empty_history ? 0.f : NAN;
      T* orow = reinterpret_cast<T*>(p.out) +
                (tok * p.num_q_heads + h * p.group + row % p.group) * 128;
      const uint32_t pv = pack2<T>(v, v);
      for (int i = 0; i < 16; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(pv, pv, pv, pv);
    }

    if (n > 0) {
      kvc += (uint32_t)n;
      tc0 += (uint32_t)n;
      if (b_active) tc1 += (uint32_t)n;
      ++qc;
    }
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
    // The last K and V loads issued complete after every earlier one.
    if (last_issued[0] >= 0) {
      const uint32_t c = (uint32_t)last_issued[0];
      mbar_wait(bar(kKFull + kslot(c)), kphase(c));
    }
    if (last_issued[1] >= 0) {
      const uint32_t c = (uint32_t)last_issued[1];
      mbar_wait(bar(kVFull + vslot(c)), vphase(c));
    }
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

int prefill_tokens_per_unit(int32_t group) { return 2 * kRows / group; }

// The kernel's registers allow a full 352-thread block on this device.
bool prefill_kernel_fits() {
  static int cached_device = -1;
  static bool fits = false;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_device) {
    cudaFuncAttributes fa_h, fa_b;
    fits = cudaFuncGetAttributes(&fa_h, paged_prefill_kernel<__half>) == cudaSuccess &&
           cudaFuncGetAttributes(&fa_b, paged_prefill_kernel<__nv_bfloat16>) == cudaSuccess &&
           fa_h.maxThreadsPerBlock >= kThreads && fa_b.maxThreadsPerBlock >= kThreads;
    cached_device = dev;
  }
  return fits;
}

bool prefill_tc_supported(const AttentionProblem& a) {
  const int group = a.num_q_heads / a.num_kv_heads;
  const int64_t num_slots = a.num_blocks * a.block_size;
  return (a.dtype == MVB_DTYPE_F16 || a.dtype == MVB_DTYPE_BF16) && a.head_dim == 128 &&
         group >= 1 && group <= 16 && (kRows % group) == 0 && (a.block_size % 16) == 0 &&
         ((uintptr_t)a.query % 16) == 0 && ((uintptr_t)a.cache % 16) == 0 &&
         ((uintptr_t)a.out % 16) == 0 && (a.q_st % 8) == 0 && (a.q_sh % 8) == 0 &&
         a.q_sh >= 128 && 2 * num_slots < ((int64_t)1 << 31) && a.num_tokens < ((int64_t)1 << 31) &&
         encoder() != nullptr && prefill_kernel_fits();
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
