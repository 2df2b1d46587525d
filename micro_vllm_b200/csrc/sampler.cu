// Batched token sampler: one launch picks the next token of every row of a
// logits matrix, on the device, with no host round trip per row.  Restates
// the per-row policy of the reference Sampler (sampling/sampler.py:39-87):
//   temperature == 0: argmax (the first index among equal maxima, as
//     torch.argmax);
//   otherwise: x = float(logit) / temperature; top-k keeps the k largest
//     (none when k <= 0 or k >= vocab; among equal values at the cut, the
//     lowest indices); top-p keeps, in descending order, every token whose
//     mass before it is <= top_p (values tied at the cut in index order);
//     one token is drawn with probability proportional to exp(x - max) over
//     the kept set.
// Division by T > 0 is monotone, so the kernel orders tokens by the logit
// itself: the same order as x, with equal x from different fp32 logits
// (impossible for fp16/bf16) ordered by the logit, then by index.  Masses
// are exp((logit - max logit) / T), computed as one FMA and exp2f per token.
// The uniform draw comes from Philox4x32-10 (Salmon, Moraes, Dror and Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by the row's
// seed with the row's sample index as counter, so a (seed, sample index)
// pair always gives the same token whatever the other rows are; the stream
// is this sampler's own, not torch's.  A row given Exp(1) noise instead
// (drawn by the caller from a generator seeded as the reference seeds its
// own) ends in the exponential race torch.multinomial runs: the kept token
// with the largest exp(x - max) / noise.
//
// One CTA of 512 threads per row; the row is read in tiles of 4096 tokens
// (16-byte loads, 8 consecutive tokens per thread, so a tile is in index
// order) and re-read from L2 by each pass.  Masses are in 1.31 fixed point: every sum is an exact integer, independent of the order of
// additions, so the top-p cut and the draw are deterministic and the draw
// always lands on a kept token.
//   pass 1: the max logit, and (top-k) a count histogram of the top 11 bits
//           of the order-preserving key of the logit;
//   top-k:  the bin holding the k-th largest key; while it holds more than
//           2048 tokens, one more histogram pass on the next digit (11, then
//           10 bits); then its tokens are gathered into shared memory and
//           bitonic-sorted (key descending, index ascending): the k-th entry
//           is the cut;
//   pass:   the total mass Z of the kept-by-k tokens and (top-p) a mass
//           histogram of their top 11 bits; the bin where the mass from the
//           top crosses top_p * Z, refined the same way, gathered and
//           sorted; a scan of the sorted masses gives the cut;
//   draw:   target = floor(u * kept mass) with a 64-bit uniform u, placed by
//           a scan of per-thread kept masses (thread-major token order) and
//           found by warp 0 among the owning thread's tokens; when the kept
//           set was sorted in shared memory, by a scan of the sorted masses.
// Top-p's mass histogram bins tokens by their distance below the max (fine,
// value-uniform bins); a bin crowded beyond kCap tokens falls back to the
// key-digit refinement.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kVec = 8;                 // consecutive tokens per thread per tile
constexpr int kTile = kThreads * kVec;  // tokens per tile
constexpr int kBins = 2048;             // 11-bit key digits
constexpr int kMassBins = 4096;         // top-p value bins
constexpr int kCap = 2048;              // boundary candidates sorted in shared memory
constexpr int kSeg = 256;               // each warp's segment of the candidate buffer
constexpr uint32_t kFull = 0xffffffffu;

// Digit levels of the 32-bit key: bits 31..21, 20..10, 9..0.
__device__ __forceinline__ int digit_shift(int level) { return level == 0 ? 21 : (level == 1 ? 10 : 0); }
__device__ __forceinline__ int digit_bins(int level) { return level == 2 ? 1024 : kBins; }
// Key bits fixed once `levels` digits are chosen.
__device__ __forceinline__ uint32_t done_mask(int levels) {
  return levels == 1 ? 0xFFE00000u : (levels == 2 ? 0xFFFFFC00u : 0xFFFFFFFFu);
}

struct SampleParams {
  const char* logits;
  int64_t row_stride;  // elements
  int64_t vocab;
  int32_t elem;  // MVB_DTYPE_*
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const uint64_t* seed;
  const int64_t* sample_index;
  int64_t* out;
  const float* noise;        // Exp(1) noise rows, or NULL
  int64_t noise_stride;      // elements between noise rows
  int32_t num_noise_rows;
  const int32_t* noise_row;  // per row: its noise row; outside [0, num_noise_rows): none
};

struct SampleSmem {
  uint32_t hist[kMassBins];
  unsigned long long mass[kMassBins];
  // (key << 32) | ~index: descending = key desc, index asc.  Warp w appends
  // to [w * kSeg, (w + 1) * kSeg); collect() compacts to [0, count).
  unsigned long long cand[kWarps * kSeg];
  unsigned long long red64[kWarps];
  float redf[kWarps];
  uint32_t ncand;
  uint32_t wcnt[kWarps];
  uint32_t sel_bin, sel_rank, sel_cnt, sel_none, sel_above_cnt, sel_lo;
  unsigned long long sel_above;
  long long found;
};

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Philox4x32-10 from the paper: 10 rounds of two 32x32 multiplies with the
// published multipliers and Weyl key increments.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// One row of logits, 8 consecutive values per call (16-byte loads when the
// row start is 16-byte aligned).
struct RowReader {
  const char* ptr;
  int64_t V;
  int32_t elem;
  bool vec;

  __device__ __forceinline__ float one(int64_t i) const {
    if (elem == MVB_DTYPE_F32) return reinterpret_cast<const float*>(ptr)[i];
    if (elem == MVB_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(ptr)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(ptr)[i]);
  }

  // Values of tokens i0 .. i0+7 (those below V); returns how many are valid.
  __device__ __forceinline__ int load(int64_t i0, float (&v)[kVec]) const {
    const int64_t left = V - i0;
    const int n = left <= 0 ? 0 : (left >= kVec ? kVec : (int)left);
    if (vec && n == kVec) {
      if (elem == MVB_DTYPE_F32) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(ptr) + (i0 >> 2));
        const float4 b = __ldg(reinterpret_cast<const float4*>(ptr) + (i0 >> 2) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
        v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
      } else {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(ptr + i0 * 2));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f;
          if (elem == MVB_DTYPE_F16) {
            __half2 h;
            memcpy(&h, &w[j], 4);
            f = __half22float2(h);
          } else {
            __nv_bfloat162 h;
            memcpy(&h, &w[j], 4);
            f = __bfloat1622float2(h);
          }
          v[2 * j] = f.x, v[2 * j + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < kVec; ++j) v[j] = j < n ? one(i0 + j) : 0.f;
    }
    return n;
  }
};

// Runs f(i0, v, n) on each of the thread's tiles in index order.  For 16-bit
// rows the 16-byte loads of four tiles are issued before any is converted,
// so four loads per thread are in flight (a pass is latency-bound otherwise).
template <class F>
__device__ __forceinline__ void for_each_tile(const RowReader& rd, int tid, F&& f) {
  constexpr int kU = 4;
  const int64_t base = (int64_t)tid * kVec;
  for (int64_t t0 = 0; t0 < rd.V; t0 += kU * kTile) {
    if (rd.vec && rd.elem != MVB_DTYPE_F32 && t0 + kU * kTile <= rd.V) {
      uint4 raw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) raw[u] = __ldg(reinterpret_cast<const uint4*>(rd.ptr + (t0 + u * kTile + base) * 2));
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        float v[kVec];
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fv;
          if (rd.elem == MVB_DTYPE_F16) {
            __half2 h;
            memcpy(&h, &w[j], 4);
            fv = __half22float2(h);
          } else {
            __nv_bfloat162 h;
            memcpy(&h, &w[j], 4);
            fv = __bfloat1622float2(h);
          }
          v[2 * j] = fv.x, v[2 * j + 1] = fv.y;
        }
        f(t0 + u * kTile + base, v, kVec);
      }
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        float v[kVec];
        const int n = rd.load(t0 + u * kTile + base, v);
        f(t0 + u * kTile + base, v, n);
      }
    }
  }
}

// Mass of a token of logit l: exp((l - lmax) / T) = 2^(l c1 - lmax c1) with
// c1 = log2(e) / T and c2 = lmax c1, in 1.31 fixed point (the max token has
// 2^31; a token below 2^-31 has none).
__device__ __forceinline__ unsigned long long mass_of(float l, float c1, float c2) {
  return __float2uint_rz(fminf(exp2f(fmaf(l, c1, -c2)), 1.0f) * 2147483648.0f);
}

// Bin of the top-p mass histogram: by distance below the max logit in steps
// of T * 22.25 / 4096 (tokens of nonzero mass lie within 21.5 T of it),
// stored so that a larger logit has a larger (or equal) bin.  Fine,
// value-uniform bins keep the histogram's shared-memory adds from piling
// onto a few addresses.  s1 = 4096 / (22.25 T).
constexpr float kMassBinScale = (float)kMassBins / 22.25f;
__device__ __forceinline__ uint32_t mass_bin(float x, float mx, float s1) {
  const float d = (mx - x) * s1;
  const uint32_t b = d < (float)(kMassBins - 1) ? __float2uint_rz(d) : (uint32_t)(kMassBins - 1);
  return (uint32_t)(kMassBins - 1) - b;
}

// Histogram adds: one shared-memory reduction per token (the hardware
// serialises lanes that hit the same bin).  Mass histograms leave out tokens
// of zero fixed-point mass (probability below 2^-32): they sit below every
// top-p cut unless top_p > 1 - vocab * 2^-32.
__device__ __forceinline__ void hist_count(uint32_t* hist, uint32_t bin, bool ok) {
  if (ok) atomicAdd(&hist[bin], 1u);
}

// Exact 64-bit add in shared memory from native 32-bit atomics: the low
// word takes v (< 2^32) and a wrap carries one into the high word (a 64-bit
// shared atomic would loop on compare-and-swap under contention).
__device__ __forceinline__ void smem_add64(unsigned long long* p, uint32_t v) {
  uint32_t* w = reinterpret_cast<uint32_t*>(p);
  const uint32_t old = atomicAdd(w, v);
  if (old + v < old) atomicAdd(w + 1, 1u);
}

__device__ __forceinline__ void hist_mass(uint32_t* hist, unsigned long long* mass, uint32_t bin, bool ok,
                                          unsigned long long m) {
  if (ok && m > 0) {
    smem_add64(&mass[bin], (uint32_t)m);
    atomicAdd(&hist[bin], 1u);
  }
}

__device__ __forceinline__ float block_max(float v, SampleSmem& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  __syncthreads();
  if (lane == 0) s.redf[warp] = v;
  __syncthreads();
  float t = lane < kWarps ? s.redf[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(kFull, t, o));
  return t;
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, SampleSmem& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(kFull, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) s.red64[warp] = v;
  __syncthreads();
  unsigned long long t = lane < kWarps ? s.red64[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(kFull, t, o);
    t = w > t ? w : t;
  }
  return t;
}

// Exclusive prefix over the block's threads (thread order) of an integer;
// *total receives the block total.  Exact.
__device__ __forceinline__ unsigned long long block_excl_scan(unsigned long long v, SampleSmem& s,
                                                              unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long u = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += u;
  }
  __syncthreads();
  if (lane == 31) s.red64[warp] = inc;
  __syncthreads();
  const unsigned long long w = lane < kWarps ? s.red64[lane] : 0ull;
  unsigned long long winc = w;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long u = __shfl_up_sync(kFull, winc, o);
    if (lane >= o) winc += u;
  }
  const unsigned long long warp_before = __shfl_sync(kFull, winc - w, warp);
  *total = __shfl_sync(kFull, winc, kWarps - 1);
  return warp_before + inc - v;
}

// Warp 0: the bin (of nbins, walked from the top) holding the rank-th
// largest counted token; publishes bin, rank within it and its count.
__device__ __forceinline__ void pick_by_rank(SampleSmem& s, int nbins, uint32_t rank) {
  const int lane = threadIdx.x & 31;
  const int per = nbins / 32;
  const int top = nbins - 1 - lane * per;  // this lane's bins: top, top-1, ..., top-per+1
  uint32_t sum = 0;
  for (int b = 0; b < per; ++b) sum += s.hist[top - b];
  uint32_t inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += u;
  }
  const uint32_t exc = inc - sum;
  const unsigned hit = __ballot_sync(kFull, exc < rank && inc >= rank);
  if (hit == 0) {  // fewer counted tokens than rank: not reached for a valid k
    if (lane == 0) {
      s.sel_bin = 0;
      s.sel_rank = 1;
      s.sel_cnt = s.hist[0];
    }
    return;
  }
  if (lane == __ffs(hit) - 1) {
    uint32_t acc = exc;
    for (int b = 0; b < per; ++b) {
      const uint32_t h = s.hist[top - b];
      if (acc + h >= rank) {
        s.sel_bin = (uint32_t)(top - b);
        s.sel_rank = rank - acc;
        s.sel_cnt = h;
        break;
      }
      acc += h;
    }
  }
}

// Warp 0: the first bin from the top where above + the mass through it
// exceeds tp; publishes bin, the mass strictly above it, its count and the
// count of the bins above it, or sel_none when the whole range stays within
// tp.
__device__ __forceinline__ void pick_by_mass(SampleSmem& s, int nbins, unsigned long long above,
                                             unsigned long long tp) {
  const int lane = threadIdx.x & 31;
  const int per = nbins / 32;
  const int top = nbins - 1 - lane * per;
  unsigned long long sum = 0;
  uint32_t csum = 0;
  for (int b = 0; b < per; ++b) {
    sum += s.mass[top - b];
    csum += s.hist[top - b];
  }
  unsigned long long inc = sum;
  uint32_t cinc = csum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long u = __shfl_up_sync(kFull, inc, o);
    const uint32_t cu = __shfl_up_sync(kFull, cinc, o);
    if (lane >= o) {
      inc += u;
      cinc += cu;
    }
  }
  const unsigned long long exc = inc - sum;
  const unsigned hit = __ballot_sync(kFull, above + exc <= tp && above + inc > tp);
  if (hit == 0) {
    if (lane == 0) s.sel_none = 1;
    return;
  }
  if (lane == __ffs(hit) - 1) {
    unsigned long long acc = above + exc;
    uint32_t cacc = cinc - csum;
    for (int b = 0; b < per; ++b) {
      const unsigned long long m = s.mass[top - b];
      if (acc + m > tp) {
        s.sel_bin = (uint32_t)(top - b);
        s.sel_above = acc;
        s.sel_cnt = s.hist[top - b];
        s.sel_above_cnt = cacc;
        break;
      }
      acc += m;
      cacc += s.hist[top - b];
    }
  }
}

// Warp 0: the range of top-p value bins that holds the cut, from per-bin
// mass bounds.  A token in the bin k places below the top (d = (max - l) *
// s1 in [k, k+1)) has mass 2^31 exp(-d / S) with S = kMassBinScale, so the
// bin's mass lies between its count times 2^31 exp(-(k+1)/S) and 2^31
// exp(-k/S) (widened for rounding).  The cut's bin is at or below the first
// bin where the upper-bound running sum passes tp, and at or above the
// first where the lower-bound sum does.  Publishes sel_bin (top bin of the
// range), sel_lo (its bottom bin), sel_above_cnt (tokens above the range),
// sel_cnt (tokens in it); sel_none when no upper-bound sum passes tp.
__device__ __forceinline__ void pick_range(SampleSmem& s, unsigned long long tp) {
  const int lane = threadIdx.x & 31;
  constexpr int per = kMassBins / 32;
  const double r = exp(-1.0 / (double)kMassBinScale);
  double hi = 2147483648.0 * exp(-(double)(lane * per) / (double)kMassBinScale);  // bound at k = lane * per
  double ub = 0, lb = 0;
  uint32_t cnt = 0;
  for (int q = 0; q < per; ++q) {
    const int k = lane * per + q;
    const uint32_t c = s.hist[kMassBins - 1 - k];
    const double lo = k == kMassBins - 1 ? 0.0 : hi * r;
    ub += (double)c * (fmin(hi, 2147483648.0) * 1.0001 + 1.0);
    lb += (double)c * fmax(lo * 0.9999 - 1.0, 0.0);
    cnt += c;
    hi *= r;
  }
  double ub_inc = ub, lb_inc = lb;
  uint32_t c_inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(kFull, ub_inc, o), l = __shfl_up_sync(kFull, lb_inc, o);
    const uint32_t c = __shfl_up_sync(kFull, c_inc, o);
    if (lane >= o) {
      ub_inc += u;
      lb_inc += l;
      c_inc += c;
    }
  }
  const double tpd = (double)tp;
  const unsigned hit_u = __ballot_sync(kFull, ub_inc > tpd);
  const unsigned hit_l = __ballot_sync(kFull, lb_inc > tpd);
  if (hit_u == 0) {
    if (lane == 0) s.sel_none = 1;
    return;
  }
  // The first bin (from the top) of the lane holding each crossing.
  const int lu = __ffs(hit_u) - 1, ll = hit_l ? __ffs(hit_l) - 1 : 31;
  if (lane == lu || lane == ll) {
    double hi2 = 2147483648.0 * exp(-(double)(lane * per) / (double)kMassBinScale);
    double u = ub_inc - ub, l = lb_inc - lb;
    uint32_t c = c_inc - cnt;
    int k_u = -1, k_l = kMassBins - 1;
    uint32_t c_above_u = 0;
    for (int q = 0; q < per; ++q) {
      const int k = lane * per + q;
      const uint32_t cc = s.hist[kMassBins - 1 - k];
      const double lo = k == kMassBins - 1 ? 0.0 : hi2 * r;
      const double nu = u + (double)cc * (fmin(hi2, 2147483648.0) * 1.0001 + 1.0);
      const double nl = l + (double)cc * fmax(lo * 0.9999 - 1.0, 0.0);
      if (k_u < 0 && nu > tpd) {
        k_u = k;
        c_above_u = c;
      }
      if (nl > tpd) {
        k_l = k;
        break;
      }
      u = nu;
      l = nl;
      c += cc;
      hi2 *= r;
    }
    if (lane == lu) {
      s.sel_bin = (uint32_t)(kMassBins - 1 - k_u);
      s.sel_above_cnt = c_above_u;
      s.sel_none = 0;
    }
    if (lane == ll) s.sel_lo = (uint32_t)(kMassBins - 1 - (hit_l ? k_l : kMassBins - 1));
  }
  __syncwarp();
  if (lane == 0) {  // tokens in the range
    uint32_t c = 0;
    for (uint32_t b = s.sel_lo; b <= s.sel_bin; ++b) c += s.hist[b];
    s.sel_cnt = c;
  }
}

// Bitonic sort of s.cand[0, n) (n a power of two, <= kCap) descending.
__device__ __forceinline__ void sort_candidates(SampleSmem& s, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = s.cand[i], b = s.cand[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            s.cand[i] = b;
            s.cand[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

__device__ __forceinline__ unsigned long long cand_of(uint32_t key, int64_t i) {
  return ((unsigned long long)key << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i);
}

__device__ __forceinline__ int64_t cand_index(unsigned long long c) {
  return (int64_t)(0xFFFFFFFFu - (uint32_t)(c & 0xFFFFFFFFull));
}

// Exponential race, the form torch.multinomial(probabilities, 1, generator)
// takes: the token that maximises p / q, q the row's Exp(1) noise drawn by
// the caller from the reference's generator.  p = exp(x - max x) with x =
// logit / T in fp32, as the reference's filtered logits; its softmax
// denominator is common to every token, so leaving it out can change the
// winner only where the two best ratios agree to within fp32 rounding.
// Packed as a candidate: the largest entry is the largest ratio, lowest
// index first, as torch.argmax.
__device__ __forceinline__ unsigned long long race_entry(float l, float temp, float xm, const float* q,
                                                         int64_t i) {
  const float x = __fdiv_rn(l, temp);
  const float r = __fdiv_rn(expf(x - xm), __ldg(q + i));
  return cand_of(order_key(r), i);
}

__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const SampleParams p) {
  extern __shared__ __align__(16) unsigned char sample_smem_raw[];
  SampleSmem& s = *reinterpret_cast<SampleSmem*>(sample_smem_raw);
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int esz = p.elem == MVB_DTYPE_F32 ? 4 : 2;
  RowReader rd;
  rd.ptr = p.logits + row * p.row_stride * esz;
  rd.V = p.vocab;
  rd.elem = p.elem;
  rd.vec = (reinterpret_cast<uintptr_t>(rd.ptr) & 15) == 0;
  const int64_t V = p.vocab;
  const float temp = p.temperature[row];

  // ---- greedy: largest value, first index among equals -----------------
  if (!(temp > 0.f)) {
    // Each thread meets its tokens in increasing index order, so a strict
    // comparison keeps the first of equal maxima.
    uint32_t bkey = 0;
    int64_t bidx = -1;
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const uint32_t k = order_key(v[j]);
        if (j < n && (bidx < 0 || k > bkey)) {
          bkey = k;
          bidx = i0 + j;
        }
      }
    });
    unsigned long long best = bidx < 0 ? 0ull : cand_of(bkey, bidx);
    best = block_max_u64(best, s);
    if (tid == 0) p.out[row] = cand_index(best);
    return;
  }

  const int32_t k_req = p.top_k[row];
  const bool use_k = k_req > 0 && (int64_t)k_req < V;
  const float top_p = p.top_p[row];
  const bool use_p = top_p < 1.f;
  // A row with noise ends in an exponential race over its kept set instead
  // of the Philox draw.
  const int32_t nrow = p.noise != nullptr ? p.noise_row[row] : -1;
  const float* qn = nrow >= 0 && nrow < p.num_noise_rows ? p.noise + (int64_t)nrow * p.noise_stride : nullptr;

  // ---- pass 1: max, and the top-k digit histogram ------------------------
  if (use_k)
    for (int b = tid; b < kBins; b += kThreads) s.hist[b] = 0;
  __syncthreads();
  float mx = -INFINITY;
  if (use_k) {
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        if (j < n) mx = fmaxf(mx, v[j]);
        hist_count(s.hist, order_key(v[j]) >> digit_shift(0), j < n);
      }
    });
  } else {
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j)
        if (j < n) mx = fmaxf(mx, v[j]);
    });
  }
  mx = block_max(mx, s);
  const float c1 = __fdiv_rn(1.4426950408889634f, temp);  // log2(e) / T
  const float c2 = mx * c1;
  const float s1 = __fdiv_rn(kMassBinScale, temp);
  const float xm = __fdiv_rn(mx, temp);  // the largest x (division by T > 0 is monotone)
  __syncthreads();

  // Index of the rank-th token (index order) whose key satisfies `hit`; used
  // only when more than kCap tokens share the exact key at a cut.
  auto nth_in_order = [&](uint32_t rank, auto hit) -> int64_t {
    unsigned long long before = 0;
    if (tid == 0) s.found = -1;
    __syncthreads();
    for (int64_t t0 = 0; t0 < V; t0 += kTile) {
      const int64_t i0 = t0 + (int64_t)tid * kVec;
      float v[kVec];
      const int n = rd.load(i0, v);
      uint32_t mine = 0;
#pragma unroll
      for (int j = 0; j < kVec; ++j)
        mine += (j < n && hit(order_key(v[j]), i0 + j)) ? 1u : 0u;
      unsigned long long total;
      const unsigned long long exc = block_excl_scan(mine, s, &total);
      if (before + exc < rank && before + exc + mine >= rank) {
        unsigned long long acc = before + exc;
        for (int j = 0; j < n; ++j) {
          if (hit(order_key(v[j]), i0 + j) && ++acc == rank) {
            s.found = i0 + j;
            break;
          }
        }
      }
      __syncthreads();
      if (s.found >= 0) break;
      before += total;
    }
    const int64_t f = s.found;
    __syncthreads();
    return f;
  };

  const uint4 r = philox4x32_10(
      make_uint4((uint32_t)p.sample_index[row], (uint32_t)((uint64_t)p.sample_index[row] >> 32), 0u, 0u),
      make_uint2((uint32_t)p.seed[row], (uint32_t)(p.seed[row] >> 32)));
  const unsigned long long u64 = ((unsigned long long)r.y << 32) | r.x;

  // ---- candidate sets in shared memory ------------------------------------
  // gather(want, positive_only) collects every token with want(x, key, i)
  // (and nonzero mass when positive_only), with its mass, and sorts them
  // (key descending, index ascending).  finish() ends the row on a sorted
  // set that starts at the largest token: its first n entries are the
  // kept-by-k tokens (all of them without top-k), top-p is a scan of their
  // masses and the draw a scan of the kept masses (in sorted order).
  // Candidates go to per-warp segments (one counter per warp, so appends
  // from different warps never contend on an address); collect() compacts
  // them through s.mass and sorts the keys.  A candidate's mass is not
  // stored: it is a function of its logit, which its key holds, so cmass(i)
  // recomputes it after the sort.  collect() returns the number of
  // candidates, or -1 when a warp overflowed its segment or they exceed kCap.
  auto seg_reset = [&]() {
    if (tid < kWarps) s.wcnt[tid] = 0;
    __syncthreads();
  };
  auto push = [&](uint32_t key, int64_t i) {
    const uint32_t slot = atomicAdd(&s.wcnt[warp], 1u);
    if (slot < (uint32_t)kSeg) s.cand[warp * kSeg + slot] = cand_of(key, i);
  };
  auto collect = [&]() -> int {
    __syncthreads();
    uint32_t total = 0, off = 0;
    bool over = false;
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c = s.wcnt[w];
      over |= c > (uint32_t)kSeg;
      if (w < warp) off += c;
      total += c;
    }
    if (over || total > (uint32_t)kCap) return -1;
    const uint32_t mine = s.wcnt[warp];
    for (uint32_t i = tid & 31; i < mine; i += 32) s.mass[off + i] = s.cand[warp * kSeg + i];
    __syncthreads();
    const int c = (int)total, n2 = pow2_at_least(c);
    for (int i = tid; i < n2; i += kThreads) s.cand[i] = i < c ? s.mass[i] : 0ull;  // pads sort last
    __syncthreads();
    sort_candidates(s, n2);
    return c;
  };
  auto cmass = [&](int i) -> unsigned long long {
    return mass_of(key_value((uint32_t)(s.cand[i] >> 32)), c1, c2);
  };
  auto gather = [&](auto want, bool positive_only) -> int {
    seg_reset();
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const float x = v[j];
        const uint32_t key = order_key(x);
        if (j < n && want(x, key, i0 + j) && (!positive_only || mass_of(x, c1, c2) > 0)) push(key, i0 + j);
      }
    });
    return collect();
  };
  constexpr int kPer = kCap / kThreads;  // consecutive sorted entries per thread
  auto finish = [&](int n, bool z_known, unsigned long long z) {
    unsigned long long mine = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      if (i < n) mine += cmass(i);
    }
    unsigned long long tot;
    const unsigned long long exc = block_excl_scan(mine, s, &tot);
    int keep = n;
    if (use_p) {
      const unsigned long long tp =
          (unsigned long long)((double)fmaxf(top_p, 0.f) * (double)(z_known ? z : tot));
      if (tid == 0) s.found = n;
      __syncthreads();
      unsigned long long acc = exc;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int i = tid * kPer + q;
        if (i < n) {
          if (acc > tp) {
            atomicMin(&s.found, (long long)i);
            break;
          }
          acc += cmass(i);
        }
      }
      __syncthreads();
      keep = (int)max(s.found, 1ll);  // the top token is always kept
    }
    if (qn != nullptr) {
      unsigned long long best = 0;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int i = tid * kPer + q;
        if (i < keep) {
          const unsigned long long e = s.cand[i];
          const unsigned long long r = race_entry(key_value((uint32_t)(e >> 32)), temp, xm, qn, cand_index(e));
          best = r > best ? r : best;
        }
      }
      best = block_max_u64(best, s);
      if (tid == 0) p.out[row] = cand_index(best);
      return;
    }
    unsigned long long kmine = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      if (i < keep) kmine += cmass(i);
    }
    unsigned long long kept_total;
    unsigned long long before = block_excl_scan(kmine, s, &kept_total);
    const unsigned long long target = __umul64hi(kept_total, u64);  // in [0, kept mass)
    if (tid == 0) p.out[row] = cand_index(s.cand[0]);  // replaced below; the top token has mass 2^31
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      if (i < keep) {
        const unsigned long long m = cmass(i);
        if (m > 0 && before <= target && target < before + m) p.out[row] = cand_index(s.cand[i]);
        before += m;
      }
    }
  };
  // The top-p cut inside a sorted candidate set of c tokens that comes right
  // below mass `above`: sorted entry i is cut when the mass before it
  // exceeds tp; the first entry is always kept (above <= tp).
  auto cut_candidates = [&](int c, unsigned long long above, unsigned long long tp, uint32_t& pk,
                            int64_t& pl) -> int {
    unsigned long long mine = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      if (i < c) mine += cmass(i);
    }
    unsigned long long tot;
    const unsigned long long exc = block_excl_scan(mine, s, &tot);
    if (tid == 0) s.found = c;
    __syncthreads();
    unsigned long long acc = above + exc;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      if (i < c) {
        if (acc > tp) {
          atomicMin(&s.found, (long long)i);
          break;
        }
        acc += cmass(i);
      }
    }
    __syncthreads();
    const int cut = max((int)s.found, 1);
    const unsigned long long e = s.cand[cut - 1];
    pk = (uint32_t)(e >> 32);
    pl = cand_index(e);
    __syncthreads();
    return cut;
  };

  if (use_k) {
    if (warp == 0) pick_by_rank(s, kBins, (uint32_t)k_req);
    __syncthreads();
    // Tokens in the boundary bin and above: k - (rank within the bin) + its count.
    if ((uint32_t)k_req - s.sel_rank + s.sel_cnt <= (uint32_t)kCap) {
      const uint32_t b = s.sel_bin;
      if (gather([&](float, uint32_t key, int64_t) { return (key >> digit_shift(0)) >= b; }, false) >= 0) {
        finish(k_req, false, 0ull);
        return;
      }
    }
    __syncthreads();
  }

  // ---- top-k cut: keep key > k_key, and key == k_key at index <= k_last ----
  uint32_t k_key = 0;
  int64_t k_last = INT64_MAX;
  if (use_k) {
    if (warp == 0) pick_by_rank(s, kBins, (uint32_t)k_req);
    __syncthreads();
    uint32_t prefix = s.sel_bin << digit_shift(0), rank = s.sel_rank, cnt = s.sel_cnt;
    int levels = 1;
    while (cnt > (uint32_t)kCap && levels < 3) {
      const int nb = digit_bins(levels), shift = digit_shift(levels);
      const uint32_t done = done_mask(levels);
      __syncthreads();
      for (int b = tid; b < nb; b += kThreads) s.hist[b] = 0;
      __syncthreads();
      for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const uint32_t key = order_key(v[j]);
          hist_count(s.hist, (key >> shift) & (uint32_t)(nb - 1), j < n && (key & done) == prefix);
        }
      });
      __syncthreads();
      if (warp == 0) pick_by_rank(s, nb, rank);
      __syncthreads();
      prefix |= s.sel_bin << shift;
      rank = s.sel_rank;
      cnt = s.sel_cnt;
      ++levels;
    }
    if (cnt > (uint32_t)kCap) {  // more than kCap tokens share the exact key
      k_key = prefix;
      k_last = nth_in_order(rank, [&](uint32_t key, int64_t) { return key == prefix; });
    } else {
      const uint32_t done = done_mask(levels);
      if (tid == 0) s.ncand = 0;
      __syncthreads();
      for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const uint32_t key = order_key(v[j]);
          if (j < n && (key & done) == prefix) {
            const uint32_t slot = atomicAdd(&s.ncand, 1u);
            if (slot < (uint32_t)kCap) s.cand[slot] = cand_of(key, i0 + j);
          }
        }
      });
      __syncthreads();
      const int c = (int)min(s.ncand, (uint32_t)kCap);
      const int n2 = pow2_at_least(c);
      for (int i = c + tid; i < n2; i += kThreads) s.cand[i] = 0ull;  // sorts last
      __syncthreads();
      sort_candidates(s, n2);
      const unsigned long long e = s.cand[rank - 1];
      k_key = (uint32_t)(e >> 32);
      k_last = cand_index(e);
      __syncthreads();
    }
  }
  auto kept_by_k = [&](uint32_t key, int64_t i) -> bool {
    return !use_k || key > k_key || (key == k_key && i <= k_last);
  };

  // ---- total mass of the kept-by-k tokens; top-p count histogram ---------
  if (use_p)
    for (int b = tid; b < kMassBins; b += kThreads) s.hist[b] = 0;
  __syncthreads();
  unsigned long long zmine = 0;
  for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const float x = v[j];
      const uint32_t key = order_key(x);
      const bool ok = j < n && kept_by_k(key, i0 + j);
      const unsigned long long m = ok ? mass_of(x, c1, c2) : 0ull;
      zmine += m;
      if (use_p) hist_count(s.hist, mass_bin(x, mx, s1), ok && m > 0);
    }
  });
  unsigned long long Z;
  const unsigned long long zexc = block_excl_scan(zmine, s, &Z);
  __syncthreads();

  // ---- top-p cut: keep key > p_key, and key == p_key at index <= p_last ----
  bool cut_p = false, have_sums = false;
  uint32_t p_key = 0;
  int64_t p_last = INT64_MAX;
  unsigned long long my_kept = zmine;  // this thread's kept mass (thread-major draw order)
  if (use_p) {
    const unsigned long long tp = (unsigned long long)((double)fmaxf(top_p, 0.f) * (double)Z);
    if (tid == 0) s.sel_none = 0;
    __syncthreads();
    if (warp == 0) pick_range(s, tp);
    __syncthreads();
    if (!s.sel_none) {
      cut_p = true;
      uint32_t b_hi = s.sel_bin, b_lo = s.sel_lo, rcnt = s.sel_cnt;
      if (!use_k && s.sel_above_cnt + rcnt <= (uint32_t)kCap) {
        // Every token of the range and above fits: finish there.
        const int c = gather([&](float x, uint32_t, int64_t) { return mass_bin(x, mx, s1) >= b_lo; }, true);
        if (c >= 0) {
          finish(c, true, Z);
          return;
        }
      }
      if (rcnt > (uint32_t)kCap) {
        // A crowded range: one pass sums the exact mass above it and of each
        // of its bins (atomics only for the range's tokens), which pins the
        // cut to one bin.
        for (uint32_t b = b_lo + tid; b <= b_hi; b += kThreads) s.mass[b] = 0ull;
        __syncthreads();
        unsigned long long above_mine = 0;
        for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
          for (int j = 0; j < kVec; ++j) {
            const float x = v[j];
            if (!(j < n && kept_by_k(order_key(x), i0 + j))) continue;
            const uint32_t vbin = mass_bin(x, mx, s1);
            if (vbin > b_hi) {
              above_mine += mass_of(x, c1, c2);
            } else if (vbin >= b_lo) {
              const unsigned long long m = mass_of(x, c1, c2);
              if (m > 0) smem_add64(&s.mass[vbin], (uint32_t)m);
            }
          }
        });
        unsigned long long above_total;
        block_excl_scan(above_mine, s, &above_total);
        if (tid == 0) {
          unsigned long long acc = above_total;
          uint32_t b = b_hi;
          while (b > b_lo && acc + s.mass[b] <= tp) acc += s.mass[b--];
          s.sel_bin = b;
          s.sel_cnt = s.hist[b];
        }
        __syncthreads();
        b_hi = b_lo = s.sel_bin;
        rcnt = s.sel_cnt;
        __syncthreads();
      }
      bool cut_done = false;
      if (rcnt <= (uint32_t)kCap) {
        // One pass: the exact mass above the range (per thread) and the
        // range's tokens into shared memory.
        seg_reset();
        unsigned long long above_mine = 0;
        for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
          for (int j = 0; j < kVec; ++j) {
            const float x = v[j];
            const uint32_t key = order_key(x);
            if (!(j < n && kept_by_k(key, i0 + j))) continue;
            const uint32_t vbin = mass_bin(x, mx, s1);
            if (vbin > b_hi) {
              above_mine += mass_of(x, c1, c2);
            } else if (vbin >= b_lo) {
              if (mass_of(x, c1, c2) > 0) push(key, i0 + j);
            }
          }
        });
        const int c = collect();
        if (c >= 0) {
          unsigned long long above_total;
          block_excl_scan(above_mine, s, &above_total);
          const int cut = cut_candidates(c, above_total, tp, p_key, p_last);
          // Each thread's kept mass: its tokens above the range plus its
          // kept range tokens (token i belongs to thread (i mod 4096) / 8).
          s.mass[tid] = 0ull;
          __syncthreads();
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const int i = tid * kPer + q;
            if (i < cut) smem_add64(&s.mass[(cand_index(s.cand[i]) & (kTile - 1)) / kVec], (uint32_t)cmass(i));
          }
          __syncthreads();
          my_kept = above_mine + s.mass[tid];
          have_sums = true;
          cut_done = true;
        }
      }
      if (!cut_done) {
        // A crowded value bin: search by key digits, refining until the
        // boundary holds at most one warp segment of tokens (so no warp
        // overflows its segment when they are gathered).
        for (int b = tid; b < kBins; b += kThreads) {
          s.hist[b] = 0;
          s.mass[b] = 0ull;
        }
        __syncthreads();
        for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
          for (int j = 0; j < kVec; ++j) {
            const float x = v[j];
            const uint32_t key = order_key(x);
            const bool ok = j < n && kept_by_k(key, i0 + j);
            hist_mass(s.hist, s.mass, key >> digit_shift(0), ok, ok ? mass_of(x, c1, c2) : 0ull);
          }
        });
        __syncthreads();
        if (tid == 0) s.sel_none = 0;
        __syncthreads();
        if (warp == 0) pick_by_mass(s, kBins, 0ull, tp);
        __syncthreads();
        uint32_t prefix = s.sel_bin << digit_shift(0), cnt = s.sel_cnt;
        unsigned long long above = s.sel_above;
        int levels = 1;
        while (cnt > (uint32_t)kSeg && levels < 3) {
          const int nb = digit_bins(levels), shift = digit_shift(levels);
          const uint32_t done = done_mask(levels);
          __syncthreads();
          for (int b = tid; b < nb; b += kThreads) {
            s.hist[b] = 0;
            s.mass[b] = 0ull;
          }
          __syncthreads();
          for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
              const float x = v[j];
              const uint32_t key = order_key(x);
              const bool ok = j < n && (key & done) == prefix && kept_by_k(key, i0 + j);
              hist_mass(s.hist, s.mass, (key >> shift) & (uint32_t)(nb - 1), ok, ok ? mass_of(x, c1, c2) : 0ull);
            }
          });
          __syncthreads();
          // Exact sums: the bin's digits hold its whole mass, so one of them
          // crosses tp again.
          if (warp == 0) pick_by_mass(s, nb, above, tp);
          __syncthreads();
          prefix |= s.sel_bin << shift;
          above = s.sel_above;
          cnt = s.sel_cnt;
          ++levels;
        }
        if (cnt > (uint32_t)kSeg) {  // more than kSeg kept tokens share the exact key
          const unsigned long long q = mass_of(key_value(prefix), c1, c2);
          unsigned long long j = q > 0 ? (tp - above) / q + 1 : (unsigned long long)cnt;
          if (j > cnt) j = cnt;
          p_key = prefix;
          p_last = nth_in_order((uint32_t)j,
                                [&](uint32_t key, int64_t i) { return key == prefix && kept_by_k(key, i); });
        } else {
          const uint32_t done = done_mask(levels);
          const int c = gather(
              [&](float, uint32_t key, int64_t i) { return (key & done) == prefix && kept_by_k(key, i); }, true);
          cut_candidates(c, above, tp, p_key, p_last);
        }
      }
    }
  }
  auto kept = [&](uint32_t key, int64_t i) -> bool {
    if (!kept_by_k(key, i)) return false;
    return !cut_p || key > p_key || (key == p_key && i <= p_last);
  };

  // ---- exponential race over the kept tokens (rows with noise) ------------
  if (qn != nullptr) {
    unsigned long long best = 0;
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const float x = v[j];
        if (j < n && kept(order_key(x), i0 + j)) {
          const unsigned long long r = race_entry(x, temp, xm, qn, i0 + j);
          best = r > best ? r : best;
        }
      }
    });
    best = block_max_u64(best, s);
    if (tid == 0) p.out[row] = cand_index(best);
    return;
  }

  // ---- draw: inverse CDF over the kept tokens, thread-major order ---------
  // The draw orders tokens by thread: thread t's tokens (tile by tile, 8 at a
  // time) before thread t+1's.  Each thread's kept mass is summed (the mass
  // pass has it already when there is no top-p cut), one scan places the
  // target in one thread, and that thread walks its own tokens.
  unsigned long long my_before = zexc, kept_total = Z;
  if (have_sums) {
    my_before = block_excl_scan(my_kept, s, &kept_total);
  } else if (cut_p) {
    my_kept = 0;
    for_each_tile(rd, tid, [&](const int64_t i0, const float (&v)[kVec], const int n) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const float x = v[j];
        if (j < n && kept(order_key(x), i0 + j)) my_kept += mass_of(x, c1, c2);
      }
    });
    my_before = block_excl_scan(my_kept, s, &kept_total);
  }
  const unsigned long long target = __umul64hi(kept_total, u64);  // in [0, kept mass)
  if (tid == 0) {
    p.out[row] = 0;  // replaced below: the largest token alone carries mass 2^31
    s.found = -1;
  }
  __syncthreads();
  if (my_kept > 0 && my_before <= target && target < my_before + my_kept) {
    s.found = tid;
    s.sel_above = my_before;
  }
  __syncthreads();
  // Warp 0 walks the owning thread's tokens, 32 of its tiles at a time.
  const int owner = (int)s.found;
  if (warp == 0 && owner >= 0) {
    const int lane = tid & 31;
    const int64_t ntiles = (V + kTile - 1) / kTile;
    unsigned long long acc = s.sel_above;
    for (int64_t r0 = 0; r0 < ntiles; r0 += 32) {
      const int64_t i0 = (r0 + lane) * kTile + (int64_t)owner * kVec;
      float v[kVec];
      const int n = r0 + lane < ntiles ? rd.load(i0, v) : 0;
      unsigned long long m[kVec], sum = 0;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const float x = v[j];
        m[j] = (j < n && kept(order_key(x), i0 + j)) ? mass_of(x, c1, c2) : 0ull;
        sum += m[j];
      }
      unsigned long long inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long u = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += u;
      }
      const unsigned long long first = acc + inc - sum;
      const bool here = first <= target && target < first + sum;
      if (here) {
        unsigned long long a2 = first;
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          a2 += m[j];
          if (m[j] > 0 && target < a2) {
            p.out[row] = i0 + j;
            break;
          }
        }
      }
      if (__any_sync(kFull, here)) break;
      acc += __shfl_sync(kFull, inc, 31);
    }
  }
}

}  // namespace

int launch_sample(const SampleArgs& a) {
  SampleParams p;
  p.logits = static_cast<const char*>(a.logits);
  p.row_stride = a.row_stride;
  p.vocab = a.vocab;
  p.elem = a.dtype;
  p.temperature = a.temperature;
  p.top_k = a.top_k;
  p.top_p = a.top_p;
  p.seed = a.seed;
  p.sample_index = a.sample_index;
  p.out = a.out_tokens;
  p.noise = a.noise;
  p.noise_stride = a.noise_stride;
  p.num_noise_rows = (int32_t)a.num_noise_rows;
  p.noise_row = a.noise_row;
  if (a.num_rows > INT32_MAX) return MVB_ERR_UNSUPPORTED_SHAPE;
  const int smem = (int)sizeof(SampleSmem);
  cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return MVB_ERR_CUDA;
  }
  sample_kernel<<<(unsigned)a.num_rows, kThreads, smem, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
