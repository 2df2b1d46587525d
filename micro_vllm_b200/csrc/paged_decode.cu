// Stream-K split-KV GQA paged decode for head_dim 128, fp16/bf16.
//
// Work decomposition.  The planner lays the KV of every decode-class
// request out as one sequence of 16-token tiles (per KV-head group of up to
// 8 heads).  The grid is persistent, one CTA per SM, and CTA b walks the
// contiguous share [b*N/G, (b+1)*N/G) of the N tiles, so every CTA moves
// the same number of bytes whatever the context-length mix.  A request
// whose tiles fall inside one share is finished by that CTA; only requests
// cut by a share boundary leave fp32 partials (at most two per CTA), which
// the CTA finishing last merges (an atomic count per request and KV head;
// no CTA ever waits for another).
//
// Inside a CTA (warp specialisation, mbarrier ring of kStages tiles):
//   * producer warp: for each tile, 16 lanes copy the 16 token rows of K
//     and 16 lanes those of V with cp.async.bulk — each row is the
//     contiguous heads_per_cta x 256 B piece of one token's cache row, so a
//     tile moves whole 2 KiB rows (one 32 KiB page per plane at 8 heads).
//     Rows outside the visible range or with an invalid page are copied
//     from a zero row, so every tile carries the same byte count.  Rows are
//     padded by 16 B in shared memory, which makes the ldmatrix reads
//     below bank-conflict free.
//   * consumer warps, one per KV head: S^T = K . Q^T with mma.sync
//     m16n8k16 (16 tokens in M; the 8 N columns hold the query heads of the
//     GQA group times the request's query tokens), fp32 online softmax with
//     3-step warp-shuffle column reductions, O^T += V^T . P^T with P moved
//     into the B-operand layout by movmatrix.trans.
// Every mbarrier wait is bounded; a wait that runs out sets
// kStatusWaitTimeout in the status word and the CTA returns.
//
// Semantics follow ReferenceAttentionOperator.forward (reference.py:14-81):
// query token t of request r sees positions
//   max(ctx_start[first token of r], ctx_start[t]) .. min(ctx_len[r]-1, pos[t]);
// softmax(q.k * scale) in fp32; empty gathered history -> 0, empty window
// -> NaN.  HBM traffic: one read of every visible K/V row (the roofline is
// HBM bandwidth).
#include <math.h>

#include <mutex>
#include <type_traits>

#include "mvb_common.cuh"
#include "mvb_internal.h"
#include "ptx_sm100.cuh"

namespace mvb {
namespace {

constexpr int kTile = 16;
constexpr int kStages = 3;
constexpr int kWin = 256;  // block-table entries the producer keeps in shared memory
constexpr int kHeadRow = kDecodeHeadDim * 2;  // bytes of one head's row
constexpr int kWaitLimit = 1 << 22;  // polls of a normal launch's waits

struct DecodeParams {
  const char* query;
  int64_t q_st_bytes, q_sh_bytes;
  char* out;
  const char* cache;
  int64_t plane_bytes;
  int64_t num_blocks;
  int64_t num_slots;  // slots per plane: value rows follow the key rows in the page map
  int32_t block_size, bs_shift, num_kv_heads, heads_per_cta, group, num_q_heads;
  const int64_t *qpos, *qstart, *qsl, *ctx_len, *table;
  int64_t table_stride, table_width, num_requests;
  float scale_log2;
  const int64_t* ctrl;
  const int64_t* tile_prefix;
  const int32_t* cta_start;
  int32_t* merge_count;
  const char* zero_row;
  float* partial_o;    // [kMaxDecodeCtas][2][8 heads][8 cols][128]
  float2* partial_ml;  // [kMaxDecodeCtas][2][8 heads][8 cols] (max, sum)
  int32_t* status;
  int32_t wait_limit;  // polls before a wait gives up
  int32_t stall_cta, stall_tile;  // test hook: that CTA's producer skips that tile (-1: none)
};

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the status bit) when the barrier never flips.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int32_t* status,
                                          int32_t limit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (status != nullptr) atomicOr(status, kStatusWaitTimeout);
  return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
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

// The visible KV extent of request r: [lo, hi) and its tile origin.
struct Extent {
  int64_t qs, lo, hi, base;
};
__device__ __forceinline__ Extent extent_of(const DecodeParams& p, int64_t r) {
  Extent e;
  e.qs = __ldg(p.qsl + r);
  e.lo = max(__ldg(p.qstart + e.qs), (int64_t)0);
  e.hi = __ldg(p.ctx_len + r);
  e.base = e.lo & ~(int64_t)15;
  return e;
}

// CTA holding global tile x when N tiles are split over G CTAs.
__device__ __forceinline__ int64_t cta_of(int64_t x, int64_t n_all, int64_t grid) {
  return ((x + 1) * grid - 1) / n_all;
}

struct Slot {  // per-stage header written by the producer
  int32_t vr;         // virtual request: group * R + r
  int32_t tile;       // tile index inside the request
  uint32_t row_mask;  // bit i: row i holds a visible, valid key
  int32_t pad;
};

// Waits (bounded) for the full barriers of the last kStages tiles issued
// before tile k, skipping none: a stage whose copy was never issued simply
// times out.
__device__ __forceinline__ void drain_issued(uint32_t full0, int k, int32_t limit) {
  for (int i = k - kStages > 0 ? k - kStages : 0; i < k; ++i)
    mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1, nullptr, limit);
}

// Polls of a wait: the constant kWaitLimit in a normal launch, the armed
// limit in the stall-hook instantiation.
template <bool kHook>
__device__ __forceinline__ int32_t wait_limit(const DecodeParams& p) {
  return kHook ? p.wait_limit : kWaitLimit;
}

// ------------------------------------------------------------ producer
// kHook: the instantiation launched only when mvb_debug_arm_decode_stall armed
// a stall (waits bounded by the armed limit, one tile skipped); normal
// launches run kHook = false.
// kPaged: a tile is one TMA load per plane through `kvmap` (block sizes
// that are multiples of 16, so a tile's 16 rows lie in one page), landing
// 128-byte swizzled; otherwise each lane copies one row with cp.async.bulk
// into 16-byte padded rows.
template <bool kHook, bool kPaged>
__device__ void produce(const DecodeParams& p, const CUtensorMap* kvmap, int64_t first,
                        int64_t last, int64_t tiles, uint8_t* ring, Slot* slots, uint32_t full0,
                        uint32_t empty0, int32_t stage_bytes, int32_t plane_stride, int32_t rowp,
                        int64_t* win) {
  const int lane = threadIdx.x & 31;
  const int hb = p.heads_per_cta;
  const int row = lane & 15, plane = lane >> 4;
  const uint32_t copy_bytes = hb * kHeadRow;
  int64_t r = __ldg(p.cta_start + blockIdx.x);
  int64_t group = first / tiles;
  Extent e = extent_of(p, r);
  int64_t req_lo = __ldg(p.tile_prefix + r), req_hi = __ldg(p.tile_prefix + r + 1);
  const int64_t* trow = p.table + r * p.table_stride;
  int64_t win_r = -1, win_lo = 0;  // request and first page held in win[]
  int k = 0;
  bool stalled = false;
  for (int64_t x = first; x < last; ++x, ++k) {
    const int64_t g = x / tiles, local = x - g * tiles;
    if (g != group || local >= req_hi) {  // next request (skip those with no tiles)
      if (g != group) {
        group = g;
        r = 0;
      }
      req_lo = __ldg(p.tile_prefix + r);
      req_hi = __ldg(p.tile_prefix + r + 1);
      while (local >= req_hi) {
        ++r;
        req_lo = req_hi;
        req_hi = __ldg(p.tile_prefix + r + 1);
      }
      e = extent_of(p, r);
      trow = p.table + r * p.table_stride;
    }
    const int64_t tile = local - req_lo;
    const int64_t pos = e.base + tile * kTile + row;
    int64_t off, lb;
    if (p.bs_shift >= 0) {
      lb = pos >> p.bs_shift;
      off = pos & (p.block_size - 1);
    } else {
      lb = pos / p.block_size;
      off = pos - lb * p.block_size;
    }
    // -2: outside the visible extent; -1: outside the table.
    const bool in_extent = pos >= e.lo && pos < e.hi;
    const bool in_table = pos >= 0 && lb < p.table_width;
    // Page lookups come from a window of the request's block table that the
    // warp loads into shared memory with coalesced loads (once per request
    // and per 256 pages), so no tile waits on a dependent global load.  A
    // paged tile needs its page whichever of its rows are visible.
    const bool need = (kPaged || in_extent) && in_table;
    if (__any_sync(0xffffffffu, need && (r != win_r || lb < win_lo || lb >= win_lo + kWin))) {
      const int64_t lo0 = __shfl_sync(0xffffffffu, lb, 0);  // row 0 holds the tile's first page
      for (int j = lane; j < kWin; j += 32) {
        const int64_t q = lo0 + j;
        win[j] = q < p.table_width ? __ldg(trow + q) : 0;
      }
      __syncwarp();
      win_r = r;
      win_lo = lo0;
    }
    const int64_t raw_blk = need ? win[lb - win_lo] : 0;  // checked after the wait
    const int s = k % kStages;
    if (!mbar_wait(empty0 + 8 * s, ((k / kStages) & 1) ^ 1, p.status, wait_limit<kHook>(p))) {
      // A consumer stopped: let the copies already issued land before the
      // CTA leaves (each wait is bounded again).
      drain_issued(full0, k, wait_limit<kHook>(p));
      return;
    }
    if (kHook && k == p.stall_tile && (int)blockIdx.x == p.stall_cta) {
      // Test hook (mvb_debug_arm_decode_stall): nothing is issued for this
      // tile, so its stage never fills and the consumers' wait for it runs
      // out; no copy is in flight for it.
      stalled = true;
      continue;
    }
    const bool page_ok = in_table && raw_blk >= 0 && raw_blk < p.num_blocks;
    const int64_t blk = !in_extent ? -2 : page_ok ? raw_blk : -1;
    const bool valid = blk >= 0;
    if (blk == -1 && p.status != nullptr) atomicOr(p.status, MVB_STATUS_BLOCK_OUT_OF_RANGE);
    const uint32_t mask = __ballot_sync(0xffffffffu, valid) & 0xffffu;
    if (lane == 0) {
      slots[s] = Slot{(int32_t)(group * p.num_requests + r), (int32_t)tile, mask, 0};
      mbar_expect_tx(full0 + 8 * s, 2 * kTile * copy_bytes);
    }
    __syncwarp();
    if constexpr (kPaged) {
      // The tile's 16 rows are slots off .. off + 15 of one page (page 0
      // stands in for a missing one; its rows are masked and zeroed).
      if (lane == 0) {
        const int64_t slot0 = (page_ok ? raw_blk : 0) * p.block_size + off;
        const uint32_t dst = smem_u32(ring + s * stage_bytes);
        const int32_t seg0 = (int32_t)(2 * group * hb);
        sm100::tma_load_3d(dst, kvmap, 0, (int32_t)slot0, seg0, full0 + 8 * s);
        sm100::tma_load_3d(dst + plane_stride, kvmap, 0, (int32_t)(p.num_slots + slot0), seg0,
                           full0 + 8 * s);
      }
      continue;
    }
    const char* src =
        valid ? p.cache + plane * p.plane_bytes +
                    ((blk * p.block_size + off) * p.num_kv_heads + group * hb) * kHeadRow
              : p.zero_row;
    bulk_g2s(smem_u32(ring + s * stage_bytes + plane * plane_stride + row * rowp), src, copy_bytes,
             full0 + 8 * s);
  }
  // The copies of the last stages have landed before the CTA may exit.  In a
  // normal launch the consumers waited for them already (the probes succeed
  // at once); after a stall the consumers left early and this drain is what
  // keeps the CTA alive until its copies are done.
  if (kHook && stalled) drain_issued(full0, k, wait_limit<kHook>(p));
}

// ------------------------------------------------------------ consumer
template <typename T, bool kHook, bool kPaged>
__device__ void consume(const DecodeParams& p, int64_t first, int64_t last, int64_t tiles,
                        int64_t n_all, const uint8_t* ring, const Slot* slots, uint32_t full0,
                        uint32_t empty0, int32_t stage_bytes, int32_t plane_stride, int32_t rowp) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int hb = p.heads_per_cta;
  const int64_t grid = gridDim.x;

  int64_t cur_vr = -1, r = 0, seg_first = 0, req_tiles = 0;
  int kvh = 0, ncols = 0;
  Extent e{0, 0, 0, 0};
  int64_t wlo[2] = {1, 1}, whi[2] = {0, 0};
  uint32_t qb[8][2];
  float m[2], l[2], o[8][4];

  int k = 0;
  for (int64_t x = first; x < last; ++x, ++k) {
    const int s = k % kStages;
    if (!mbar_wait(full0 + 8 * s, (k / kStages) & 1, p.status, wait_limit<kHook>(p))) return;
    const Slot slot = slots[s];
    if (slot.vr != cur_vr) {  // a new request segment starts in this CTA
      cur_vr = slot.vr;
      const int64_t grp = cur_vr / p.num_requests;
      r = cur_vr - grp * p.num_requests;
      kvh = (int)grp * hb + w;
      e = extent_of(p, r);
      ncols = (int)(__ldg(p.qsl + r + 1) - e.qs) * p.group;
      req_tiles = __ldg(p.tile_prefix + r + 1) - __ldg(p.tile_prefix + r);
      seg_first = slot.tile;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int n = 2 * c + j;
        if (n < ncols) {
          const int64_t t = e.qs + n / p.group;
          wlo[j] = max(e.lo, __ldg(p.qstart + t));
          whi[j] = min(e.hi - 1, __ldg(p.qpos + t));
        } else {
          wlo[j] = 1;
          whi[j] = 0;
        }
      }
      if (g < ncols) {
        const int64_t t = e.qs + g / p.group;
        const int hq = kvh * p.group + g % p.group;
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
      m[0] = m[1] = -INFINITY;
      l[0] = l[1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }

    // ---- one 16-token tile of KV head kvh ----
    // The tile's K and V fragments go to registers first, and the stage is
    // released before any math: the producer refills it while this warp
    // computes, so a stage is held for the 16 loads, not the whole tile.
    uint32_t ka[8][4], va[8][4];
    if constexpr (kPaged) {
      // Plane layout: [2 hb segments of 64 elements][16 rows][128 B], each
      // 128-byte row with its 16-byte chunks XOR-swizzled by (row & 7), so
      // the 8 rows of an ldmatrix read fall in 8 different bank groups.
      // This warp's head owns segments 2w (dims 0-63) and 2w + 1.
      const uint32_t kb = smem_u32(ring + s * stage_bytes) + (uint32_t)(2 * w * kTile * 128);
      const uint32_t vb = kb + plane_stride;
      if (slot.row_mask != 0xffffu) {
        // Rows no query may see hold stale bytes of the page (or a stand-in
        // page): zero their values so 0 x NaN cannot reach O.
        uint8_t* vrows = const_cast<uint8_t*>(ring) + s * stage_bytes + plane_stride + 2 * w * kTile * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = lane + 32 * j;  // (half, row, chunk) = (i / 128, i / 8 % 16, i % 8)
          const int row = (i >> 3) & 15;
          if (!((slot.row_mask >> row) & 1u))
            *reinterpret_cast<uint4*>(vrows + (i >> 7) * kTile * 128 + row * 128 + (i & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        sm100::fence_proxy_async();  // ordered before the next TMA write of this stage
        __syncwarp();
      }
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int chunk = 2 * (ks & 3) + (lane >> 4);
        ldsm_x4(kb + (uint32_t)(((ks >> 2) * kTile + row) * 128 + ((chunk ^ (row & 7)) << 4)), ka[ks]);
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int row = (lane & 7) + (lane >> 4) * 8;
        const int chunk = 2 * (mt & 3) + ((lane >> 3) & 1);
        ldsm_x4_t(vb + (uint32_t)(((mt >> 2) * kTile + row) * 128 + ((chunk ^ (row & 7)) << 4)), va[mt]);
      }
    } else {
      const uint32_t kb = smem_u32(ring + s * stage_bytes) + w * kHeadRow;
      const uint32_t vb = kb + plane_stride;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4(kb + row * rowp + (2 * ks + (lane >> 4)) * 16, ka[ks]);
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int row = (lane & 7) + (lane >> 4) * 8;
        ldsm_x4_t(vb + row * rowp + (2 * mt + ((lane >> 3) & 1)) * 16, va[mt]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);  // release: orders the loads above first
    // Two accumulators halve the dependent chain of the 8 k-steps.
    float sc[4] = {0.f, 0.f, 0.f, 0.f}, sc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      if (ks & 1)
        mma16816<T>(sc2, ka[ks], qb[ks][0], qb[ks][1]);
      else
        mma16816<T>(sc, ka[ks], qb[ks][0], qb[ks][1]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] += sc2[i];
    const int64_t p0 = e.base + (int64_t)slot.tile * kTile + g, p1 = p0 + 8;
    const bool ok0 = (slot.row_mask >> g) & 1u, ok1 = (slot.row_mask >> (g + 8)) & 1u;
    // Online softmax with a lazily moved reference: m[j] (the column's
    // running max) moves only when a score exceeds it by more than 2^8, so
    // most tiles need neither the column-max shuffles nor a rescale of O.
    // O and l share the reference, so O / l is exact whatever it is, and
    // P <= 2^8 stays well inside fp16 / bf16.
    float sv[4], pr[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      sv[j] = (ok0 && p0 >= wlo[j] && p0 <= whi[j]) ? sc[j] * p.scale_log2 : -INFINITY;
      sv[2 + j] = (ok1 && p1 >= wlo[j] && p1 <= whi[j]) ? sc[2 + j] * p.scale_log2 : -INFINITY;
    }
    const bool jump = sv[0] > m[0] + 8.f || sv[2] > m[0] + 8.f || sv[1] > m[1] + 8.f || sv[3] > m[1] + 8.f;
    if (__any_sync(0xffffffffu, jump)) {
      float corr[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float tmax = fmaxf(sv[j], sv[2 + j]);
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
        const float mn = fmaxf(m[j], tmax);
        corr[j] = exp2f(m[j] - (mn == -INFINITY ? 0.f : mn));
        l[j] *= corr[j];
        m[j] = mn;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= corr[0];
        o[mt][1] *= corr[1];
        o[mt][2] *= corr[0];
        o[mt][3] *= corr[1];
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float mu = m[j] == -INFINITY ? 0.f : m[j];
      pr[j] = exp2f(sv[j] - mu);
      pr[2 + j] = exp2f(sv[2 + j] - mu);
      l[j] += pr[j] + pr[2 + j];
    }
    const uint32_t ph0 = pack2<T>(pr[0], pr[1]), ph1 = pack2<T>(pr[2], pr[3]);
    const uint32_t pb0 = movmatrix_t(ph0);
    const uint32_t pb1 = movmatrix_t(ph1);
    // bf16 keeps 8 mantissa bits: P = P_hi + P_lo (both bf16) and a second
    // P.V product restore ~16 bits, matching the fp16 path's accuracy.
    constexpr bool kSplitP = std::is_same<T, __nv_bfloat16>::value;
    uint32_t pl0 = 0, pl1 = 0;
    if constexpr (kSplitP) {
      const float2 h0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ph0));
      const float2 h1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ph1));
      pl0 = movmatrix_t(pack2<T>(pr[0] - h0.x, pr[1] - h0.y));
      pl1 = movmatrix_t(pack2<T>(pr[2] - h1.x, pr[3] - h1.y));
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      mma16816<T>(o[mt], va[mt], pb0, pb1);
      if constexpr (kSplitP) mma16816<T>(o[mt], va[mt], pl0, pl1);
    }

    // ---- end of this CTA's segment of the request ----
    const bool req_done = slot.tile == req_tiles - 1;
    if (!req_done && x != last - 1) continue;
    float lsum[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v = l[j];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      lsum[j] = v;
    }
    const bool empty_history = e.hi <= e.lo;
    if (seg_first == 0 && req_done) {  // whole request in this CTA: write O / l
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int n = 2 * c + j;
        if (n >= ncols) continue;
        const float inv = lsum[j] > 0.f ? 1.f / lsum[j] : NAN;
        const int64_t t = e.qs + n / p.group;
        const int hq = kvh * p.group + n % p.group;
        T* orow = reinterpret_cast<T*>(p.out) + (t * p.num_q_heads + hq) * kDecodeHeadDim;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          orow[16 * mt + g] = from_float<T>(empty_history ? 0.f : o[mt][j] * inv);
          orow[16 * mt + g + 8] = from_float<T>(empty_history ? 0.f : o[mt][2 + j] * inv);
        }
      }
      continue;
    }
    // Partial: slot 0 when this request is the first one of the CTA's share.
    const int pslot = (seg_first == slot.tile - (x - first)) ? 0 : 1;
    const int64_t pidx = ((int64_t)blockIdx.x * 2 + pslot) * kMaxHeadsPerCta + w;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = 2 * c + j;
      float* po = p.partial_o + (pidx * kDecodeCols + n) * kDecodeHeadDim;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        po[16 * mt + g] = o[mt][j];
        po[16 * mt + g + 8] = o[mt][2 + j];
      }
      if (g == 0) p.partial_ml[pidx * kDecodeCols + n] = make_float2(m[j], lsum[j]);
    }
    __threadfence();
    __syncwarp();
    int done = 0;
    if (lane == 0) done = atomicAdd(p.merge_count + r * p.num_kv_heads + kvh, 1);
    done = __shfl_sync(0xffffffffu, done, 0);
    const int64_t grp = cur_vr / p.num_requests;
    const int64_t g0 = grp * tiles + __ldg(p.tile_prefix + r);
    const int64_t g1 = g0 + req_tiles;
    const int64_t b_first = cta_of(g0, n_all, grid), b_last = cta_of(g1 - 1, n_all, grid);
    // Segments = CTAs in [b_first, b_last] with a non-empty share (shares
    // are empty only when there are fewer tiles than CTAs).
    int nseg = 0;
    for (int64_t b = b_first; b <= b_last; ++b)
      nseg += (b * n_all / grid) < ((b + 1) * n_all / grid);
    if (done != nseg - 1) continue;
    // Every segment has counted: the counter goes back to zero for the next
    // launch over the same plan.
    if (lane == 0) p.merge_count[r * p.num_kv_heads + kvh] = 0;
    // Last segment to finish: merge all segments of (request, kvh).  The
    // segments' (max, sum) pairs are loaded one per lane and combined with
    // shuffles; the partial O rows are then read several at a time, so the
    // merge costs a few L2 round trips rather than two per segment.
    __threadfence();
    // Partial slot of CTA b for this request: 0 when it is the first request
    // of b's share, else 1.
    auto partial_index = [&](int64_t b) -> int64_t {
      const int64_t bstart = b * n_all / grid;
      const int64_t bfirst_vr = (bstart / tiles) * p.num_requests + __ldg(p.cta_start + b);
      return (b * 2 + (bfirst_vr == cur_vr ? 0 : 1)) * kMaxHeadsPerCta + w;
    };
    auto non_empty = [&](int64_t b) { return (b * n_all / grid) < ((b + 1) * n_all / grid); };
    const int64_t nb = b_last - b_first + 1;
    if (nb * ncols <= 32) {
      // Common case: every (segment, column) pair fits one lane, so all the
      // (max, sum) pairs and then all the partial rows are loaded at once.
      const int nbi = (int)nb;
      const int s_l = lane % nbi, n_l = lane / nbi;  // this lane's pair
      const int64_t b_l = b_first + s_l;
      const bool live = n_l < ncols && non_empty(b_l);
      const int64_t idx_l = live ? partial_index(b_l) : 0;
      float2 ml = make_float2(-INFINITY, 0.f);
      if (live) ml = __ldcg(&p.partial_ml[idx_l * kDecodeCols + n_l]);
      float mx_l = -INFINITY;  // max over this lane's column
      for (int k = 0; k < nbi; ++k)
        mx_l = fmaxf(mx_l, __shfl_sync(0xffffffffu, ml.x, min(n_l, ncols - 1) * nbi + k));
      const float f_l = live ? exp2f(ml.x - (mx_l == -INFINITY ? 0.f : mx_l)) : 0.f;
      float sum_l = 0.f;  // sum over this lane's column
      for (int k = 0; k < nbi; ++k) {
        const int src = min(n_l, ncols - 1) * nbi + k;
        sum_l += __shfl_sync(0xffffffffu, ml.y * f_l, src);
      }
      for (int n = 0; n < ncols; ++n) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int k = 0; k < nbi; ++k) {
          const int src = n * nbi + k;
          const float fk = __shfl_sync(0xffffffffu, f_l, src);
          const int64_t ik = __shfl_sync(0xffffffffu, idx_l, src);
          const float4 v = fk != 0.f ? __ldcg(reinterpret_cast<const float4*>(
                                               p.partial_o + (ik * kDecodeCols + n) * kDecodeHeadDim) +
                                           lane)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
          acc.x += v.x * fk;
          acc.y += v.y * fk;
          acc.z += v.z * fk;
          acc.w += v.w * fk;
        }
        const float sum = __shfl_sync(0xffffffffu, sum_l, n * nbi);
        const float inv = sum > 0.f ? 1.f / sum : NAN;
        const int64_t t = e.qs + n / p.group;
        const int hq = kvh * p.group + n % p.group;
        T* orow = reinterpret_cast<T*>(p.out) + (t * p.num_q_heads + hq) * kDecodeHeadDim + 4 * lane;
        orow[0] = from_float<T>(empty_history ? 0.f : acc.x * inv);
        orow[1] = from_float<T>(empty_history ? 0.f : acc.y * inv);
        orow[2] = from_float<T>(empty_history ? 0.f : acc.z * inv);
        orow[3] = from_float<T>(empty_history ? 0.f : acc.w * inv);
      }
      continue;
    }
    for (int n = 0; n < ncols; ++n) {
      // Pass 1: the reference max over the segments.
      float mx = -INFINITY;
      for (int64_t b0 = b_first; b0 <= b_last; b0 += 32) {
        const int64_t b = b0 + lane;
        if (b <= b_last && non_empty(b))
          mx = fmaxf(mx, __ldcg(&p.partial_ml[partial_index(b) * kDecodeCols + n].x));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mu = mx == -INFINITY ? 0.f : mx;
      // Pass 2: weighted sums; lane k of each group of 32 segments holds
      // segment k's weight and partial index.
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float sum = 0.f;
      for (int64_t b0 = b_first; b0 <= b_last; b0 += 32) {
        const int64_t b = b0 + lane;
        float f = 0.f;
        int64_t idx = 0;
        if (b <= b_last && non_empty(b)) {
          idx = partial_index(b);
          const float2 ml = __ldcg(&p.partial_ml[idx * kDecodeCols + n]);
          f = exp2f(ml.x - mu);
          sum += ml.y * f;
        }
        const int cnt = (int)min((int64_t)32, nb - (b0 - b_first));
        for (int k0 = 0; k0 < cnt; k0 += 4) {
          float4 v[4];
          float fk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = min(k0 + u, cnt - 1);
            fk[u] = k0 + u < cnt ? __shfl_sync(0xffffffffu, f, k) : 0.f;
            const int64_t ik = __shfl_sync(0xffffffffu, idx, k);
            v[u] = fk[u] != 0.f ? __ldcg(reinterpret_cast<const float4*>(
                                          p.partial_o + (ik * kDecodeCols + n) * kDecodeHeadDim) +
                                      lane)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc.x += v[u].x * fk[u];
            acc.y += v[u].y * fk[u];
            acc.z += v[u].z * fk[u];
            acc.w += v[u].w * fk[u];
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float inv = sum > 0.f ? 1.f / sum : NAN;
      const int64_t t = e.qs + n / p.group;
      const int hq = kvh * p.group + n % p.group;
      T* orow = reinterpret_cast<T*>(p.out) + (t * p.num_q_heads + hq) * kDecodeHeadDim + 4 * lane;
      orow[0] = from_float<T>(empty_history ? 0.f : acc.x * inv);
      orow[1] = from_float<T>(empty_history ? 0.f : acc.y * inv);
      orow[2] = from_float<T>(empty_history ? 0.f : acc.z * inv);
      orow[3] = from_float<T>(empty_history ? 0.f : acc.w * inv);
    }
  }
}

template <typename T, bool kHook, bool kPaged>
__global__ void __launch_bounds__(32 * (kMaxHeadsPerCta + 1), 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kvmap, const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t ring_raw[];
  // Swizzled TMA destinations want 1024-byte alignment (the launch adds the slack).
  uint8_t* ring = kPaged ? reinterpret_cast<uint8_t*>(
                               (reinterpret_cast<uintptr_t>(ring_raw) + 1023) & ~(uintptr_t)1023)
                         : ring_raw;
  __shared__ __align__(8) uint64_t bars[2 * kStages];
  __shared__ Slot slots[kStages];
  __shared__ int64_t table_win[kWin];
  const int hb = p.heads_per_cta;
  const int32_t rowp = kPaged ? hb * kHeadRow : hb * kHeadRow + 16;
  const int32_t plane_stride = kTile * rowp;
  const int32_t stage_bytes = 2 * plane_stride;
  const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[kStages]);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, hb);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  // Launched as a programmatic dependent of the planner: everything above
  // overlaps its tail; nothing the planner writes is read before this wait.
  // The prefill pass that follows may then launch as SMs free up.
  grid_dependency_wait();
  allow_dependent_launch();
  __syncthreads();
  const int64_t tiles = p.ctrl[kCtrlTiles];
  const int64_t n_all = tiles * (p.num_kv_heads / hb);
  const int64_t grid = gridDim.x;
  const int64_t first = (int64_t)blockIdx.x * n_all / grid;
  const int64_t last = ((int64_t)blockIdx.x + 1) * n_all / grid;
  if (first >= last) return;
  const int warp = threadIdx.x >> 5;
  if (warp == hb) {
    produce<kHook, kPaged>(p, &kvmap, first, last, tiles, ring, slots, full0, empty0, stage_bytes,
                           plane_stride, rowp, table_win);
  } else {
    consume<T, kHook, kPaged>(p, first, last, tiles, n_all, ring, slots, full0, empty0, stage_bytes,
                              plane_stride, rowp);
  }
}

// The dynamic shared-memory limit is a property of the kernel function on a
// device, shared by every heads-per-CTA configuration: it is always set to
// the largest ring (kMaxHeadsPerCta), so a launch with a smaller ring never
// lowers it below what a larger one needs.
int set_up(const void* fn, int smem, int threads, int* per_sm) {
  constexpr int kLargestRing = kStages * 2 * kTile * (kMaxHeadsPerCta * kHeadRow + 16);
  cudaError_t e =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kLargestRing);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, fn, threads, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return MVB_ERR_CUDA;
  }
  return MVB_OK;
}

}  // namespace

// The stall armed by mvb_debug_arm_decode_stall for this host thread's next
// decode launch.
struct StallHook {
  int32_t cta = -1, tile = -1, wait_limit = 0;
};
thread_local StallHook g_stall;

int arm_decode_stall(int32_t cta, int32_t tile, int32_t wait_limit) {
  g_stall = wait_limit > 0 ? StallHook{cta, tile, wait_limit} : StallHook{};
  return MVB_OK;
}

int heads_per_cta(int32_t num_kv_heads) {
  for (int hb = kMaxHeadsPerCta; hb > 1; --hb)
    if (num_kv_heads % hb == 0) return hb;
  return 1;
}

// The kernel's instantiations: dtype x stall hook x paged (TMA) tiles.
using DecodeKernel = void (*)(const CUtensorMap, const DecodeParams);
template <typename T>
DecodeKernel kernel_for(bool hook, bool paged) {
  return hook ? (paged ? paged_decode_kernel<T, true, true> : paged_decode_kernel<T, true, false>)
              : (paged ? paged_decode_kernel<T, false, true> : paged_decode_kernel<T, false, false>);
}
const void* const* kernel_instances() {
  static const void* fns[8] = {
      reinterpret_cast<const void*>(kernel_for<__half>(false, false)),
      reinterpret_cast<const void*>(kernel_for<__half>(false, true)),
      reinterpret_cast<const void*>(kernel_for<__half>(true, false)),
      reinterpret_cast<const void*>(kernel_for<__half>(true, true)),
      reinterpret_cast<const void*>(kernel_for<__nv_bfloat16>(false, false)),
      reinterpret_cast<const void*>(kernel_for<__nv_bfloat16>(false, true)),
      reinterpret_cast<const void*>(kernel_for<__nv_bfloat16>(true, false)),
      reinterpret_cast<const void*>(kernel_for<__nv_bfloat16>(true, true)),
  };
  return fns;
}

int decode_grid(const AttentionProblem& a, int* smem_bytes) {
  const int hb = heads_per_cta(a.num_kv_heads);
  const int smem = kStages * 2 * kTile * (hb * kHeadRow + 16);
  const int threads = 32 * (hb + 1);
  // Per device and heads-per-CTA, filled under a lock (host threads driving
  // different devices may call at the same time); the kernel attributes are
  // set on each device the first time it is seen.
  static std::mutex lock;
  static int cached[kMaxDevices][kMaxHeadsPerCta + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool slot = dev >= 0 && dev < kMaxDevices;
  std::lock_guard<std::mutex> guard(lock);
  if (!slot || cached[dev][hb] == 0) {
    // Every instantiation gets the attribute; the grid follows the lowest
    // occupancy among them (one CTA per SM for every head count here).
    int per_sm = 1 << 30;
    const void* const* fns = kernel_instances();
    for (int i = 0; i < 8; ++i) {
      int n = 0;
      if (set_up(fns[i], smem, threads, &n) != MVB_OK) return -1;
      per_sm = n < per_sm ? n : per_sm;
    }
    if (per_sm < 1) per_sm = 1;
    int grid = num_sms() * per_sm;
    grid = grid < kMaxDecodeCtas ? grid : kMaxDecodeCtas;
    if (!slot) {
      *smem_bytes = smem;
      return grid;
    }
    cached[dev][hb] = grid;
  }
  *smem_bytes = smem;
  return cached[dev][hb];
}

int launch_paged_decode(const AttentionProblem& a, const WorkspaceLayout& w, int32_t grid,
                        int32_t smem_bytes) {
  char* ws = static_cast<char*>(a.workspace);
  DecodeParams dp;
  dp.query = static_cast<const char*>(a.query);
  dp.q_st_bytes = a.q_st * 2;
  dp.q_sh_bytes = a.q_sh * 2;
  dp.out = static_cast<char*>(a.out);
  dp.cache = static_cast<const char*>(a.cache);
  dp.plane_bytes = a.num_blocks * a.block_size * (int64_t)a.num_kv_heads * kHeadRow;
  dp.num_blocks = a.num_blocks;
  dp.block_size = a.block_size;
  dp.bs_shift = (a.block_size & (a.block_size - 1)) == 0 ? __builtin_ctz(a.block_size) : -1;
  dp.num_kv_heads = a.num_kv_heads;
  dp.heads_per_cta = heads_per_cta(a.num_kv_heads);
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
  dp.ctrl = reinterpret_cast<const int64_t*>(ws + w.ctrl);
  dp.tile_prefix = reinterpret_cast<const int64_t*>(ws + w.tile_prefix);
  dp.cta_start = reinterpret_cast<const int32_t*>(ws + w.cta_start);
  dp.merge_count = reinterpret_cast<int32_t*>(ws + w.merge_count);
  dp.zero_row = ws + w.zero_row;
  dp.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
  dp.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
  dp.status = a.status;
  dp.wait_limit = kWaitLimit;
  dp.stall_cta = dp.stall_tile = -1;
  const bool hook = g_stall.wait_limit > 0;
  if (hook) {  // one-shot test hook armed on this host thread
    dp.wait_limit = g_stall.wait_limit;
    dp.stall_cta = g_stall.cta;
    dp.stall_tile = g_stall.tile;
    g_stall = StallHook{};
  }
  const int threads = 32 * (dp.heads_per_cta + 1);
  if (a.dtype != MVB_DTYPE_F16 && a.dtype != MVB_DTYPE_BF16) return MVB_ERR_UNSUPPORTED_DTYPE;
  // Paged tiles (one TMA load per plane and tile) when a tile's 16 rows lie
  // in one page and the map's 32-bit slot coordinate reaches both planes.
  // The map views the cache as [2 * slots][2 * Hkv segments][64 elements]:
  // a box of {64, 16 slots, 2 hb segments} is one tile of the CTA's heads,
  // laid out segment-major in shared memory.
  CUtensorMap kvmap{};
  bool paged = false;
  dp.num_slots = a.num_blocks * a.block_size;
  EncodeTiled encode = tensor_map_encoder();
  if (encode != nullptr && (a.block_size % kTile) == 0 && 2 * dp.num_slots < ((int64_t)1 << 31) &&
      ((uintptr_t)a.cache % 16) == 0) {
    const cuuint64_t dims[3] = {64, (cuuint64_t)(2 * dp.num_slots), (cuuint64_t)(2 * a.num_kv_heads)};
    const cuuint64_t strides[2] = {(cuuint64_t)a.num_kv_heads * kHeadRow, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)kTile, (cuuint32_t)(2 * dp.heads_per_cta)};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = a.dtype == MVB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    paged = encode(&kvmap, dt, 3, const_cast<void*>(a.cache), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (paged) smem_bytes = kStages * 2 * kTile * dp.heads_per_cta * kHeadRow + 1024;
  const DecodeKernel fn = a.dtype == MVB_DTYPE_F16 ? kernel_for<__half>(hook, paged)
                                                   : kernel_for<__nv_bfloat16>(hook, paged);
  // A programmatic dependent of the planner launched just before it.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, kvmap, dp);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return MVB_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace mvb
