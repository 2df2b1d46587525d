// Varlen causal chunked-prefill attention over the paged cache on the
// 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128, fp16/bf16.
//
// Work item = (prefill-class request, pair of 128-row query tiles, KV head).
// Each tile's 128 MMA rows are 128/G query tokens x the G query heads of one
// GQA group; the two tiles (A: the earlier tokens, B: the next ones) share
// every K/V tile fetched.  A persistent grid (one CTA per SM, 225 KB of
// shared memory, all 512 TMEM columns) pulls items from an atomic cursor,
// the query tiles with the most keys first.
//
// Roles inside a CTA (12 warps), each running its own loop over the items
// with no block-wide barrier between items, so the next item's loads and
// first MMAs overlap the current item's last tiles and epilogue:
//   warp 11  scheduler: claims the next item, computes its description
//           (request, tokens, KV head, the union of its rows' key windows
//           and so the KV tiles to visit), publishes it in a 2-slot ring and
//           loads the item's Q tiles (a 3-D tensor map over [token, head,
//           dim] so the G heads of a token land in adjacent rows), each into
//           its tile's buffer once the previous item's epilogue released it.
//   warps 8, 10  TMA producers of K and V: per 128-key KV tile, the 8 pages
//           (a 2-D tensor map over the cache's [2*NB*bs slots, Hkv*128]
//           view; one 16-row x 64-element box per page, plane and half)
//           into a 2-stage K ring and a 3-stage V ring, 128-byte swizzled —
//           the layout the tensor cores read.  Pages missing from the block
//           table are fetched from page 0 and masked.  Warp 10 then zeroes
//           the rows of each landed V tile that no query of the pair may see
//           (stale or sentinel bytes must not reach O as 0 * NaN) before the
//           P.V MMAs may read it.
//   warp 9  MMA issuer (one thread), ping-pong between the tiles:
//             S_A(0), S_B(0); then per KV tile j:
//             PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)
//           S_X = Q_X.K^T lands in TMEM (128 fp32 columns per tile); the
//           softmax writes P_X back over S_X as packed 16-bit pairs and
//           PV_X: O_X += P_X.V_j reads it straight from TMEM (A operand in
//           TMEM, V from shared memory MN-major).  tcgen05 operations of one
//           thread complete in issue order, so S_X(j+1) finishing implies
//           PV_X(j) finished, and the next item's S_X(0) runs after this
//           item's PV_X.
//   warps 0-3 / 4-7  softmax of tile A / B, one thread per row (= TMEM
//           lane): pass 1 loads the 128 scores and takes the masked max;
//           the reference max moves only when the tile max exceeds it by
//           2^8, and then O_X is rescaled in TMEM (no wait needed: O_X holds
//           PV_X(j-1), complete since S_X(j) is); pass 2 computes
//           P = 2^(s - max) from the same registers and stores it to TMEM.
//           bf16 P is split into P_hi + P_lo (two MMAs) to keep ~16 bits.
//           At the end
//           each row's O is normalised and staged in the tile's Q buffer
//           (every S of the item is done with it) for two TMA stores; the
//           next item's first P.V (which overwrites O_X) waits for this
//           warp's next P, so it cannot start before these loads.
// The softmax warpgroups (warps 0-7) raise their register limit to 200 and
// the other warpgroup (warps 8-11) lowers its own to 96, which fits in the
// 168 per thread the block is launched with (the host checks that count).
// Every mbarrier wait is bounded; a timeout sets kStatusWaitTimeout and the
// kernel winds down.
//
// Semantics are those of ReferenceAttentionOperator.forward
// (reference.py:14-81), as in the decode kernel: token t of request r sees
// max(ctx_start[first token of r], ctx_start[t]) .. min(ctx_len[r]-1, pos[t]).
// Roofline: tensor cores; algorithmic flops per request = 4 * D * Hq *
// (visible query-key pairs).
#include <math.h>

#include <mutex>

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
constexpr int kThreads = 384;               // 12 warps
constexpr int kKProdWarp = 8, kMmaWarp = 9, kSchedWarp = 11;  // warp 10: V producer
constexpr int kItemSlots = 2;
constexpr int kItemReaders = 11;            // warps 0-10 each take every item once
// Register split between the softmax warpgroups and the rest (setmaxnreg):
// 2 x 128 x 200 + 128 x 96 <= 384 x 168, the registers of the launch.
constexpr int kLaunchRegs = 168, kSoftmaxRegs = 200, kOtherRegs = 96;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * kLaunchRegs,
              "register split must fit the launch's registers");
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S/P of tile A and B, then O of tile A and B.
__device__ __forceinline__ uint32_t col_s(int t) { return 128u * (uint32_t)t; }
__device__ __forceinline__ uint32_t col_o(int t) { return 256u + 128u * (uint32_t)t; }
constexpr float kRescaleLog2 = 8.f;

// mbarrier indices, derived from the ring depths so no two overlap.
enum Bar : int {
  kQFull = 0,                           // +tile: Q tile landed
  kQEmpty = kQFull + 2,                 // +tile: the tile's epilogue is done with its Q buffer
  kKFull = kQEmpty + 2,                 // +K slot: K tile landed
  kKEmpty = kKFull + kKStages,          // +K slot: every S MMA read it
  kVFull = kKEmpty + kKStages,          // +V slot: V tile landed
  kVEmpty = kVFull + kVStages,          // +V slot: every P.V MMA read it
  kVReady = kVEmpty + kVStages,         // +V slot: the V producer fixed the tile up
  kSFull = kVReady + kVStages,          // +tile (A, B)
  kPFull = kSFull + 2,                  // +tile
  kPvDone = kPFull + 2,                 // +tile
  kOStaged = kPvDone + 2,               // +tile: the 4 warps staged O for the TMA store
  kItemFull = kOStaged + 2,             // +item slot: description written
  kItemEmpty = kItemFull + kItemSlots,  // +item slot: every reader copied it
  kFinal = kItemEmpty + kItemSlots,     // last MMA commit before TMEM is released
  kNumBars = kFinal + 1,
};
static_assert(kNumBars == 4 + 2 * kKStages + 3 * kVStages + 4 * 2 + 2 * kItemSlots + 1,
              "mbarrier layout");

// One work item as the scheduler warp describes it.
struct ItemDesc {
  int64_t q0;         // first token of tile A
  int64_t qe;         // end of the request's tokens
  int64_t gather_lo;  // first position of the request's gathered history
  int64_t clen;       // context length of the request
  int32_t r;          // request; -1 = no more items
  int32_t h;          // KV head
  int32_t n;          // KV tiles to visit (0: no row sees any key)
  int32_t kbase;      // first key of KV tile 0 (16-aligned)
  int32_t kv_lo;      // union of the rows' windows
  int32_t kv_hi;
  int32_t ntiles;     // query tiles holding rows (1 or 2)
  int32_t pad;
};

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
  const int32_t* unit_order;   // units, most keys first
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

// 12 warps: each SM sub-partition holds 3 of them, so a thread may use at
// most 168 registers (16 K registers per sub-partition).
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kvmap,
                         const __grid_constant__ CUtensorMap omap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kNumBars];
  __shared__ __align__(16) ItemDesc items[kItemSlots];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int32_t first_claim;
  __shared__ int32_t abort_sh;
  __shared__ int32_t last_issued[2];  // last K and last V tile index issued
  __shared__ int32_t q_issued[2];     // Q loads issued per tile (phases of kQFull)

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Launched as a programmatic dependent of the decode kernel, which may
  // still run: this CTA waits for it before anything else, so the pass's
  // completion implies the decode kernel's (later work reads both outputs).
  grid_dependency_wait();
  const int64_t n_items = p.ctrl[kCtrlPrefillUnits] * p.num_kv_heads;

  if (tid == 0) first_claim = atomicAdd(p.cursor, 1);
  __syncthreads();
  if (first_claim >= n_items) return;  // no prefill work for this CTA

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_addr(smem);
  const uint32_t bar0 = smem_addr(&bars[0]);
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  volatile int32_t* abort_flag = &abort_sh;

  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kQFull + t), 1);
      mbar_init(bar(kQEmpty + t), 1);
    }
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar(kKFull + s), 1);
      mbar_init(bar(kKEmpty + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(bar(kVFull + s), 1);
      mbar_init(bar(kVEmpty + s), 1);
      mbar_init(bar(kVReady + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kSFull + s), 1);
      mbar_init(bar(kPFull + s), 4);
      mbar_init(bar(kPvDone + s), 1);
      mbar_init(bar(kOStaged + s), 4);
    }
    for (int s = 0; s < kItemSlots; ++s) {
      mbar_init(bar(kItemFull + s), 1);
      mbar_init(bar(kItemEmpty + s), kItemReaders);
    }
    mbar_init(bar(kFinal), 1);
    mbar_init_fence();
    abort_sh = 0;
    last_issued[0] = last_issued[1] = -1;
    q_issued[0] = q_issued[1] = 0;
  }
  if (warp == kMmaWarp) tmem_alloc(smem_addr(&tmem_base_sh), kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  // Item i's description, copied into d (false on a timeout); each reader
  // warp releases the slot as soon as it holds its copy.
  auto take_item = [&](uint32_t i, ItemDesc& d) -> bool {
    const uint32_t slot = i % kItemSlots;
    if (!__all_sync(0xffffffffu, mbar_wait(bar(kItemFull + slot), (i / kItemSlots) & 1)))
      return false;
    d = items[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(kItemEmpty + slot));
    return true;
  };
  // Running counts (identical in every role): KV tiles of this CTA (ring
  // phases), KV tiles processed per query tile (S/P/PV phases), Q loads per
  // query tile.
  uint32_t kvc = 0, tc0 = 0, tc1 = 0, qc0 = 0, qc1 = 0;
  auto advance = [&](const ItemDesc& d) {
    if (d.n > 0) {
      kvc += (uint32_t)d.n;
      tc0 += (uint32_t)d.n;
      ++qc0;
      if (d.ntiles == 2) {
        tc1 += (uint32_t)d.n;
        ++qc1;
      }
    }
  };
  auto fail = [&]() {
    if (lane == 0) atomicOr(&abort_sh, 1);
  };

  // Each role runs its whole item loop inside its own branch, after its
  // register limit changed.
  if (warp >= kKProdWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kOtherRegs));
    if (warp == kSchedWarp) {
      // ---------------------------------------------------- scheduler
      int64_t claimed = first_claim;
      for (uint32_t i = 0;; ++i) {
        const uint32_t slot = i % kItemSlots;
        // The slot's previous description (item i-2) was copied by every reader.
        if (!__all_sync(0xffffffffu,
                        mbar_wait(bar(kItemEmpty + slot), ((i / kItemSlots) & 1) ^ 1))) {
          if (lane == 0) atomicOr(&abort_sh, 1);
          break;
        }
        if (i > 0) {
          int64_t c = 0;
          if (lane == 0) c = atomicAdd(p.cursor, 1);
          claimed = __shfl_sync(0xffffffffu, c, 0);
        }
        ItemDesc d;
        d.r = -1;
        d.pad = 0;
        if (claimed < n_items && *abort_flag == 0) {
          // Units come longest first (the planner's order), the KV heads of
          // a unit as consecutive claims.
          d.h = (int32_t)(claimed % p.num_kv_heads);
          const int64_t unit = __ldg(p.unit_order + claimed / p.num_kv_heads);
          const int32_t r = __ldg(p.unit_req + unit);
          const int64_t qt = unit - __ldg(p.unit_prefix + r);
          const int64_t qs = __ldg(p.qsl + r), qe = __ldg(p.qsl + r + 1);
          d.r = r;
          d.q0 = qs + qt * 2 * p.block_q;
          d.qe = qe;
          d.ntiles = d.q0 + p.block_q < qe ? 2 : 1;
          d.gather_lo = max(__ldg(p.qstart + qs), (int64_t)0);
          d.clen = __ldg(p.ctx_len + r);
          // Union of the windows of the pair's tokens (positions fit 32 bits:
          // the planner refuses contexts longer than 2^30).
          int32_t lo = INT32_MAX, hi = -1;
          const int64_t tend = min(d.q0 + 2 * (int64_t)p.block_q, qe);
          for (int64_t t = d.q0 + lane; t < tend; t += 32) {
            const int32_t lt = (int32_t)min(max(d.gather_lo, __ldg(p.qstart + t)), (int64_t)kMaxContext);
            const int32_t ht = (int32_t)max(min(d.clen - 1, __ldg(p.qpos + t)), (int64_t)-1);
            if (lt <= ht) {
              lo = min(lo, lt);
              hi = max(hi, ht);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
          }
          const bool any = lo != INT32_MAX;
          d.kv_lo = any ? lo : 0;
          d.kv_hi = any ? hi : -1;
          d.kbase = d.kv_lo & ~15;
          d.n = any ? (d.kv_hi - d.kbase) / kKeys + 1 : 0;
        }
        if (lane == 0) {
          items[slot] = d;
          mbar_arrive(bar(kItemFull + slot));  // release: the description is visible
        }
        __syncwarp();
        if (d.r < 0) break;
        if (d.n > 0) {
          // The item's Q tiles, each into its tile's buffer once the previous
          // user of that buffer (an earlier item's epilogue) released it.
          bool qok = true;
          if (lane == 0) {
            for (int t = 0; t < d.ntiles; ++t) {
              const uint32_t qn = t == 0 ? qc0 : qc1;
              if (!mbar_wait(bar(kQEmpty + t), (qn & 1) ^ 1)) {
                qok = false;
                break;
              }
              mbar_expect_tx(bar(kQFull + t), kTileBytes);
              const int32_t qy = d.h * p.group, qz = (int32_t)(d.q0 + (int64_t)t * p.block_q);
              tma_load_3d(sb + kOffQ + t * kTileBytes, &qmap, 0, qy, qz, bar(kQFull + t));
              tma_load_3d(sb + kOffQ + t * kTileBytes + kHalf, &qmap, 64, qy, qz, bar(kQFull + t));
              q_issued[t] = (int32_t)qn + 1;
            }
          }
          if (__shfl_sync(0xffffffffu, qok ? 1 : 0, 0) == 0) {
            if (lane == 0) atomicOr(&abort_sh, 1);
            break;
          }
          advance(d);
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------ MMA issuer
      if (lane == 0) {
        const uint32_t idesc_qk = f16_idesc(kBf16, false, kRows, kKeys);
        const uint32_t idesc_pv = f16_idesc(kBf16, true, kRows, 128);
        // Matrix descriptors of the operand buffers, built once: an operand
        // slice k bytes into a buffer adds k >> 4 to the start-address field
        // (shared memory lies below 256 KB, so the 14-bit field never carries
        // into the next one).
        const uint64_t dq0 = sw128_desc(sb + kOffQ, 16, 1024);
        const uint64_t dk0 = sw128_desc(sb + kOffK, 16, 1024);
        const uint64_t dv0 = sw128_desc(sb + kOffV, kHalf, 1024);
        auto issue_s = [&](int t, uint32_t stage) {
          const uint64_t dq = dq0 + (uint64_t)(((uint32_t)t * kTileBytes) >> 4);
          const uint64_t dk = dk0 + (uint64_t)((stage * kTileBytes) >> 4);
          const uint32_t d_tmem = tmem + col_s(t);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            constexpr uint32_t kStep[8] = {0, 2, 4, 6, kHalf >> 4, (kHalf >> 4) + 2,
                                           (kHalf >> 4) + 4, (kHalf >> 4) + 6};
            umma_f16(d_tmem, dq + kStep[k], dk + kStep[k], idesc_qk, k > 0);
          }
          umma_commit(bar(kSFull + t));
        };
        auto issue_pv = [&](int t, uint32_t stage, bool acc) {
          const uint64_t dv = dv0 + (uint64_t)((stage * kTileBytes) >> 4);
          const uint32_t d_tmem = tmem + col_o(t), p_tmem = tmem + col_s(t);
          const uint32_t idesc = idesc_pv;
#pragma unroll
          for (int part = 0; part < (kBf16 ? 2 : 1); ++part) {  // P_hi (+ P_lo in bf16)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t pcol = 32 * (k >> 1) + 8 * (k & 1) + 16 * part;
              umma_f16_ts(d_tmem, p_tmem + pcol, dv + (uint64_t)(k * (2048 >> 4)), idesc,
                          acc || k > 0 || part > 0);
            }
          }
          umma_commit(bar(kPvDone + t));
        };
        // The next item with KV tiles (items without any skip the MMAs),
        // taken by this thread alone; false at the end or on a timeout.
        uint32_t next_i = 0;
        bool ok = true;
        auto next_item = [&](ItemDesc& d) -> bool {
          for (;;) {
            const uint32_t slot = next_i % kItemSlots;
            if (!mbar_wait(bar(kItemFull + slot), (next_i / kItemSlots) & 1)) {
              ok = false;
              return false;
            }
            d = items[slot];
            mbar_arrive(bar(kItemEmpty + slot));
            ++next_i;
            if (d.r < 0 || *abort_flag != 0) return false;
            if (d.n > 0) return true;
          }
        };
        ItemDesc cur;
        while (ok && next_item(cur)) {
          const int n = cur.n, ntiles = cur.ntiles;
          // S(0) of each tile once its Q and the item's first K tile landed.
          // Barrier probes cost ~170 cycles each and the tensor pipe queues
          // only a couple of MMAs, so independent probes go out together.
          {
            bool rk, rqa, rqb;
            mbar_test3(bar(kKFull + kslot(kvc)), kphase(kvc), bar(kQFull), qc0 & 1,
                       bar(kQFull + 1), qc1 & 1, rk, rqa, rqb);
            ok = (rk || mbar_wait(bar(kKFull + kslot(kvc)), kphase(kvc))) &&
                 (rqa || mbar_wait(bar(kQFull), qc0 & 1));
            if (ok) {
              tc_fence_after();
              issue_s(0, kslot(kvc));
              if (ntiles == 2) {
                ok = rqb || mbar_wait(bar(kQFull + 1), qc1 & 1);
                if (ok) {
                  tc_fence_after();
                  issue_s(1, kslot(kvc));
                }
              }
            }
          }
          if (!ok) break;
          umma_commit(bar(kKEmpty + kslot(kvc)));  // K(0) read by every S(0)
          for (int j = 0; ok && j < n; ++j) {
            const uint32_t c = kvc + j, sv = vslot(c);
            const uint32_t cn = c + 1, skn = kslot(cn);
            const bool more = j + 1 < n;
            bool k_ready = true;
            for (int t = 0; t < ntiles; ++t) {
              const uint32_t pphase = ((t == 0 ? tc0 : tc1) + j) & 1;
              if (t == 0) {
                // P_A(j), V(j) and K(j+1) probed together.
                bool rp, rv, rk;
                mbar_test3(bar(kPFull), pphase, bar(kVReady + sv), vphase(c),
                           more ? bar(kKFull + skn) : bar(kPFull), more ? kphase(cn) : pphase, rp,
                           rv, rk);
                ok = (rp || mbar_wait(bar(kPFull), pphase)) &&
                     (rv || mbar_wait(bar(kVReady + sv), vphase(c)));
                k_ready = rk;
              } else {
                ok = mbar_wait(bar(kPFull + t), pphase);
              }
              if (!ok) break;
              tc_fence_after();
              issue_pv(t, sv, j > 0);
              if (t == ntiles - 1) umma_commit(bar(kVEmpty + sv));  // V(j) read by every P.V(j)
              if (more) {
                if (t == 0 && !k_ready) {
                  ok = mbar_wait(bar(kKFull + skn), kphase(cn));
                  if (!ok) break;
                  tc_fence_after();
                }
                issue_s(t, skn);
                if (t == ntiles - 1) umma_commit(bar(kKEmpty + skn));  // K(j+1) read by every S
              }
            }
          }
          if (!ok) break;
          advance(cur);
        }
        if (!ok) atomicOr(&abort_sh, 1);
      }
      __syncwarp();
    } else {
      // ------------------------------------------------ producers
      for (uint32_t i = 0;; ++i) {
        ItemDesc d;
        if (!take_item(i, d)) {
          fail();
          break;
        }
        if (d.r < 0 || *abort_flag != 0) break;
        const int n = d.n;
        const int64_t* trow = p.table + (int64_t)d.r * p.table_stride;
        bool ok = true;
        if (n > 0) {
          // Warp 8 loads the K tiles, warp 10 the V tiles; each waits
          // only on its own ring, so K is never held up behind a V slot.
          const bool is_k = warp == kKProdWarp;
          for (int j = 0; ok && j < n; ++j) {
            const uint32_t c = kvc + j;
            const uint32_t slot_kv = is_k ? kslot(c) : vslot(c);
            const uint32_t full = bar((is_k ? kKFull : kVFull) + slot_kv);
            // K(j) reuses the slot of K(j-2), free once every S(j-2) MMA ran;
            // V(j) that of V(j-3), free once every P.V(j-3) MMA ran.
            const uint32_t empty_phase = (is_k ? kphase(c) : vphase(c)) ^ 1;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(bar((is_k ? kKEmpty : kVEmpty) + slot_kv), empty_phase))) {
              ok = false;
              break;
            }
            const int64_t pos = (int64_t)d.kbase + (int64_t)j * kKeys + 16 * lane;
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
              const int32_t xk = d.h * 128;
              const uint32_t dst = sb + (is_k ? kOffK : kOffV) + slot_kv * kTileBytes + lane * 2048;
              tma_load_2d(dst, &kvmap, xk, y, full);
              tma_load_2d(dst + kHalf, &kvmap, xk + 64, y, full);
            }
            if (!is_k) {
              // V(c) landed: zero the rows no query of the pair may see (they
              // hold stale or sentinel bytes that must not reach O as 0 * NaN;
              // only the first and last tile and missing pages have any), then
              // release the tile to the P.V MMAs.  Lane l walks rows 4i + l/8
              // at 16-byte chunk l%8: conflict-free.
              const uint32_t pok = __ballot_sync(0xffffffffu, lane < 8 && blk >= 0) & 0xffu;
              if (j == 0 || j == n - 1 || pok != 0xffu) {
                if (!__all_sync(0xffffffffu, mbar_wait(full, vphase(c)))) {
                  ok = false;
                  break;
                }
                uint8_t* vt = smem + kOffV + slot_kv * kTileBytes;
                const int32_t k0 = d.kbase + j * kKeys;
#pragma unroll 4
                for (int it = 0; it < 32; ++it) {
                  const int row = 4 * it + (lane >> 3), cc = lane & 7;
                  const int32_t key = k0 + row;
                  if (key < d.kv_lo || key > d.kv_hi || !((pok >> (row >> 4)) & 1u)) {
                    *reinterpret_cast<uint4*>(vt + row * 128 + cc * 16) = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4*>(vt + kHalf + row * 128 + cc * 16) = make_uint4(0, 0, 0, 0);
                  }
                }
                fence_proxy_async();  // visible to the P.V MMAs
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kVReady + slot_kv));
              } else if (lane == 0) {
                // Nothing to fix: the tile is ready once it lands.
                if (!mbar_wait(full, vphase(c))) ok = false;
                mbar_arrive(bar(kVReady + slot_kv));
              }
              if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
              }
            }
          }
          ok = __all_sync(0xffffffffu, ok);
        }
        if (!ok) {
          fail();
          break;
        }
        advance(d);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------ softmax / epilogue of tile x
    // Tile 0 (A) for warps 0-3, 1 (B) for 4-7.
    const int x = warp >= 4 ? 1 : 0;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane of this thread
    uint32_t oc = 0;                         // staged epilogues of this tile (kOStaged phases)
    for (uint32_t i = 0;; ++i) {
      ItemDesc d;
      if (!take_item(i, d)) {
        fail();
        break;
      }
      if (d.r < 0 || *abort_flag != 0) break;
      const int n = d.n;
      const int ntiles = d.ntiles;
      const int64_t* trow = p.table + (int64_t)d.r * p.table_stride;
      bool ok = true;
      // Per-row visibility window (softmax threads own rows).
      const int64_t tok = d.q0 + (int64_t)x * p.block_q + row / p.group;
      const bool row_valid = tok < min(d.qe, d.q0 + (int64_t)(x + 1) * p.block_q);
      T* orow = reinterpret_cast<T*>(p.out) +
                (tok * p.num_q_heads + (int64_t)d.h * p.group + row % p.group) * 128;
      if (n == 0) {
        // No visible key at all: 0 for an empty gathered history, else NaN
        // (softmax over an all -inf row), as the reference.
        if (row_valid) {
          const float v = d.clen <= d.gather_lo ? 0.f : NAN;
          const uint32_t pv = pack2<T>(v, v);
          for (int e = 0; e < 16; ++e) reinterpret_cast<uint4*>(orow)[e] = make_uint4(pv, pv, pv, pv);
        }
      } else if (x < ntiles) {
        int32_t lo_q = 1, hi_q = 0;
        if (row_valid) {
          lo_q = (int32_t)min(max(d.gather_lo, __ldg(p.qstart + tok)), (int64_t)kMaxContext);
          hi_q = (int32_t)max(min(d.clen - 1, __ldg(p.qpos + tok)), (int64_t)-1);
        }
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t s_cols = tmem + lane_base + col_s(x);
        const uint32_t o_cols = tmem + lane_base + col_o(x);
        const uint32_t tcx = x == 0 ? tc0 : tc1;
        float m_ref = -INFINITY, l = 0.f;
        // Pages of a KV tile that exist in the block table: lanes 0-7 look
        // up one 16-key page each, one tile ahead, so the load's latency
        // hides behind the previous tile's softmax.
        int64_t blk_next = -1;
        if (lane < 8) blk_next = page_of(p, trow, (int64_t)d.kbase + 16 * lane);
        for (int j = 0; j < n; ++j) {
          const uint32_t c = kvc + j, sv = vslot(c);
          const int32_t k0 = d.kbase + j * kKeys;
          const uint32_t pok = __ballot_sync(0xffffffffu, blk_next >= 0) & 0xffu;
          blk_next = -1;
          if (lane < 8 && j + 1 < n) blk_next = page_of(p, trow, (int64_t)k0 + kKeys + 16 * lane);
          if (!__all_sync(0xffffffffu, mbar_wait(bar(kSFull + x), (tcx + j) & 1))) {
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
            for (int e = 0; e < kKeys; e += 2)
              mx[(e >> 1) & 3] = fmax3(mx[(e >> 1) & 3], __uint_as_float(sc[e >> 5][e & 31]),
                                       __uint_as_float(sc[e >> 5][(e & 31) + 1]));
          } else {
            // Visible keys as one bit per key (window [lo_rel, hi_rel) and
            // pages present), so each score needs a bit test and a select.
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              const int a0 = min(max(lo_rel - 32 * ch, 0), 32), b0 = min(max(hi_rel - 32 * ch, 0), 32);
              const uint32_t below_b = b0 >= 32 ? 0xffffffffu : ((1u << b0) - 1u);
              const uint32_t below_a = a0 >= 32 ? 0xffffffffu : ((1u << a0) - 1u);
              const uint32_t pages = (((pok >> (2 * ch)) & 1u) ? 0x0000ffffu : 0u) |
                                     (((pok >> (2 * ch + 1)) & 1u) ? 0xffff0000u : 0u);
              const uint32_t vis = below_b & ~below_a & pages;
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float va = (vis >> i) & 1u ? __uint_as_float(sc[ch][i]) : -INFINITY;
                const float vb = (vis >> (i + 1)) & 1u ? __uint_as_float(sc[ch][i + 1]) : -INFINITY;
                sc[ch][i] = __float_as_uint(va);
                sc[ch][i + 1] = __float_as_uint(vb);
                mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], va, vb);
              }
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
              for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
              tmem_st16(o_cols + 16 * ch, o);
            }
          }
          // P = 2^(s*scale - m_ref), written over S as packed 16-bit pairs:
          // keys 32ch..32ch+31 -> columns 32ch..32ch+15 (P_hi) and
          // 32ch+16..32ch+31 (P_lo, bf16 only), behind the scores already read.
          const float mu = m_ref == -INFINITY ? 0.f : m_ref;
          // Pairs of keys go through the packed fp32 pipe: s*scale - mu in
          // one fma.f32x2, the row sum in add.f32x2 accumulators.
          const uint64_t scale2 = f32x2_pack(p.scale_log2, p.scale_log2);
          const uint64_t negmu2 = f32x2_pack(-mu, -mu);
          uint64_t ps2[2] = {f32x2_pack(0.f, 0.f), f32x2_pack(0.f, 0.f)};
          // P as packed 16-bit pairs; bf16 P as P_hi + P_lo (columns
          // 32ch..+15 and 32ch+16..+31).
          {
            constexpr bool kSplit = kBf16;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {  // 16 keys: 8 packed columns per store
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const int k = 16 * hh + 2 * e;
                  float xa, xb;
                  f32x2_unpack(f32x2_fma(f32x2_pack(__uint_as_float(sc[ch][k]),
                                                    __uint_as_float(sc[ch][k + 1])),
                                         scale2, negmu2),
                               xa, xb);
                  const float pa = ex2(xa), pb = ex2(xb);
                  ps2[e & 1] = f32x2_add(ps2[e & 1], f32x2_pack(pa, pb));
                  hi[e] = pack2<T>(pa, pb);
                  if constexpr (kSplit) {
                    const float2 hf =
                        __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hi[e]));
                    lo[e] = pack2<T>(pa - hf.x, pb - hf.y);
                  }
                }
                tmem_st8(s_cols + 32 * ch + 8 * hh, hi);
                if constexpr (kSplit) tmem_st8(s_cols + 32 * ch + 16 + 8 * hh, lo);
              }
            }
          }
          tmem_wait_st();
          {
            float s0, s1, s2, s3;
            f32x2_unpack(ps2[0], s0, s1);
            f32x2_unpack(ps2[1], s2, s3);
            l += (s0 + s1) + (s2 + s3);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kPFull + x));
        }
        ok = __all_sync(0xffffffffu, ok);
        // ---- epilogue: O / l -> output rows ----
        if (ok && __all_sync(0xffffffffu, mbar_wait(bar(kPvDone + x), (tcx + n - 1) & 1))) {
          tc_fence_after();
          const float inv = l > 0.f ? 1.f / l : NAN;
          // The whole row of O in one batch of TMEM loads.
          uint32_t o[4][32];
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tmem_ld32_raw(o_cols + 32 * ch, o[ch]);
          tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) reg_fence(o[ch]);
          // 8 normalised outputs (columns 8c..8c+7) as one 16-byte vector.
          auto out8 = [&](int cchunk) {
            const float* f = reinterpret_cast<const float*>(&o[cchunk >> 2][8 * (cchunk & 3)]);
            uint4 q;
            q.x = pack2<T>(f[0] * inv, f[1] * inv);
            q.y = pack2<T>(f[2] * inv, f[3] * inv);
            q.z = pack2<T>(f[4] * inv, f[5] * inv);
            q.w = pack2<T>(f[6] * inv, f[7] * inv);
            return q;
          };
          if (d.q0 + (int64_t)(x + 1) * p.block_q <= d.qe) {
            // Every row belongs to the request: stage the tile in its own Q
            // buffer (every S of the item is done with it) in the layout of
            // the output tensor map's box and write it with two TMA stores.
            uint8_t* qbuf = smem + kOffQ + x * kTileBytes;
#pragma unroll
            for (int cchunk = 0; cchunk < 16; ++cchunk) {
              const int hf = cchunk >> 3, cc = cchunk & 7;
              *reinterpret_cast<uint4*>(qbuf + hf * kHalf + row * 128 + ((cc ^ (row & 7)) << 4)) =
                  out8(cchunk);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kOStaged + x));
            if (row == 0) {
              if (mbar_wait(bar(kOStaged + x), oc & 1)) {
                const int32_t qy = d.h * p.group, qz = (int32_t)(d.q0 + (int64_t)x * p.block_q);
                tma_store_3d(&omap, sb + kOffQ + x * kTileBytes, 0, qy, qz);
                tma_store_3d(&omap, sb + kOffQ + x * kTileBytes + kHalf, 64, qy, qz);
                bulk_commit_group();
                bulk_wait_read_all();
                mbar_arrive(bar(kQEmpty + x));  // the buffer may take the next Q
              } else {
                ok = false;
              }
            }
            ++oc;
          } else {
            // A ragged last tile: only its valid rows are stored.
            if (row_valid) {
#pragma unroll
              for (int cchunk = 0; cchunk < 16; ++cchunk)
                *reinterpret_cast<uint4*>(orow + 8 * cchunk) = out8(cchunk);
            }
            if (row == 0) mbar_arrive(bar(kQEmpty + x));
          }
        } else {
          ok = false;
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        fail();
        break;
      }
      advance(d);
    }
    if (row == 0) bulk_wait_all();  // this tile's output stores are complete
  }

  // Everything this CTA issued lands before TMEM and shared memory go away
  // (each wait bounded): the MMA thread waits on a final commit; after an
  // abort, the producers also wait for their last TMA loads.
  if (warp == kMmaWarp && lane == 0) {
    umma_commit(bar(kFinal));
    mbar_wait(bar(kFinal), 0);
  }
  __syncthreads();
  if (abort_sh && tid == 0) {
    if (p.status != nullptr) atomicOr(p.status, kStatusWaitTimeout);
    // The last K and V loads issued complete after every earlier one.
    if (last_issued[0] >= 0) {
      const uint32_t c = (uint32_t)last_issued[0];
      mbar_wait(bar(kKFull + kslot(c)), kphase(c));
    }
    if (last_issued[1] >= 0) {
      const uint32_t c = (uint32_t)last_issued[1];
      mbar_wait(bar(kVFull + vslot(c)), vphase(c));
    }
    for (int t = 0; t < 2; ++t)
      if (q_issued[t] > 0) mbar_wait(bar(kQFull + t), (q_issued[t] - 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------ host side
EncodeTiled encoder() { return tensor_map_encoder(); }

}  // namespace

EncodeTiled tensor_map_encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  });
  return fn;
}

namespace {

// Per-device host state of the prefill kernel, filled under one lock (host
// threads driving different devices may call at the same time).
struct PrefillDeviceState {
  bool checked = false, fits = false, configured = false;
};
std::mutex g_prefill_lock;
PrefillDeviceState g_prefill_state[kMaxDevices];

}  // namespace

int prefill_tokens_per_unit(int32_t group) { return 2 * kRows / group; }

// The kernel's registers allow a full 384-thread block on this device, and
// it was built with exactly the per-thread count its register split assumes.
bool prefill_kernel_fits() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> guard(g_prefill_lock);
  PrefillDeviceState& st = g_prefill_state[dev];
  if (!st.checked) {
    cudaFuncAttributes fa_h, fa_b;
    st.fits = cudaFuncGetAttributes(&fa_h, paged_prefill_kernel<__half>) == cudaSuccess &&
              cudaFuncGetAttributes(&fa_b, paged_prefill_kernel<__nv_bfloat16>) == cudaSuccess &&
              fa_h.maxThreadsPerBlock >= kThreads && fa_b.maxThreadsPerBlock >= kThreads &&
              fa_h.numRegs == kLaunchRegs && fa_b.numRegs == kLaunchRegs;
    st.checked = true;
  }
  return st.fits;
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

  CUtensorMap qmap, kvmap, omap;
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
    // The output [token, head, dim] (contiguous), boxed like Q.
    const cuuint64_t dims[3] = {128, (cuuint64_t)a.num_q_heads, (cuuint64_t)a.num_tokens};
    const cuuint64_t strides[2] = {(cuuint64_t)128 * 2, (cuuint64_t)a.num_q_heads * 128 * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(kRows / group)};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&omap, dt, 3, a.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
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
  pp.unit_order = reinterpret_cast<const int32_t*>(ws + w.prefill_unit_order);
  pp.status = a.status;

  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return MVB_ERR_INVALID_ARGUMENT;
  {
    std::lock_guard<std::mutex> guard(g_prefill_lock);
    PrefillDeviceState& st = g_prefill_state[dev];
    if (!st.configured) {
      cudaError_t e = cudaFuncSetAttribute(paged_prefill_kernel<__half>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(paged_prefill_kernel<__nv_bfloat16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return MVB_ERR_CUDA;
      }
      st.configured = true;
    }
  }
  // A programmatic dependent of the decode kernel launched just before it:
  // its CTAs take SMs as decode CTAs leave (each waits for the whole decode
  // grid first), so the launch overlaps the decode kernel's tail.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_sms());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = a.dtype == MVB_DTYPE_BF16
                            ? cudaLaunchKernelEx(&cfg, paged_prefill_kernel<__nv_bfloat16>, qmap, kvmap, omap, pp)
                            : cudaLaunchKernelEx(&cfg, paged_prefill_kernel<__half>, qmap, kvmap, omap, pp);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return MVB_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace mvb
