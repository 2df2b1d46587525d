// Batched token sampler: one launch picks the next token of every row of a
// logits matrix, on the device, with no host round trip per row.  Restates
// the per-row policy of the reference Sampler (sampling/sampler.py:39-87):
//   temperature == 0: argmax (the first index among equal maxima, as
//     torch.argmax);
//   otherwise: x = float(logit) / temperature; top-k keeps the k largest
//     (none when k <= 0 or k >= vocab; among equal values at the cut, the
//     lowest indices); top-p keeps the shortest run of tokens in descending
//     order whose mass before each token is <= top_p (values tied at the cut
//     in index order); one token is drawn with probability proportional to
//     exp(x - max) over the kept set.
// The uniform draw comes from Philox4x32-10 (Salmon, Moraes, Dror and Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by the row's
// seed with the row's sample index as counter, so a (seed, sample index)
// pair always gives the same token whatever the other rows are; the stream
// is this sampler's own, not torch's.
//
// One CTA of 1024 threads per row.  The k-th largest value and the top-p
// boundary come from a most-significant-digit radix search over the
// order-preserving 32-bit keys of the scaled logits (4 passes of 8 bits with
// shared-memory histograms of counts, and of probability mass for top-p);
// the row is re-read from L2 on each pass.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "mvb_common.cuh"
#include "mvb_internal.h"

namespace mvb {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kWarpsPerCta = kSampleThreads / 32;

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
};

__device__ __forceinline__ float load_logit(const SampleParams& p, const char* row, int64_t i) {
  if (p.elem == MVB_DTYPE_F32) return reinterpret_cast<const float*>(row)[i];
  if (p.elem == MVB_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(row)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[i]);
}

// Order-preserving key of a float: larger float -> larger unsigned key.
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
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

template <typename V>
__device__ __forceinline__ V block_sum(V v, V* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  V t = lane < kWarpsPerCta ? sh[lane] : V(0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleParams p) {
  __shared__ uint32_t hist_count[256];
  __shared__ unsigned long long hist_mass[256];  // fixed point, 2^-40 units: order-free sums
  __shared__ float red_f[kWarpsPerCta];
  __shared__ unsigned long long red_u[kWarpsPerCta];
  __shared__ float chunk_mass[kSampleThreads];
  __shared__ int64_t chunk_last[kSampleThreads];  // last kept index of each thread's chunk
  __shared__ uint32_t sel_prefix_sh, sel_rank_sh;
  __shared__ float sel_mass_sh;
  __shared__ int64_t pick_sh;

  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const char* logits = p.logits + row * p.row_stride * (p.elem == MVB_DTYPE_F32 ? 4 : 2);
  const int64_t V = p.vocab;
  const float temp = p.temperature[row];

  // ---- greedy: largest value, first index among equals -----------------
  if (!(temp > 0.f)) {
    unsigned long long best = 0ull;  // (key << 32) | ~index: max picks the lowest index
    for (int64_t i = tid; i < V; i += kSampleThreads) {
      const float x = load_logit(p, logits, i);
      const unsigned long long cand =
          ((unsigned long long)order_key(x) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i);
      best = cand > best ? cand : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) red_u[warp] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = red_u[0];
      for (int w = 1; w < kWarpsPerCta; ++w) b = red_u[w] > b ? red_u[w] : b;
      p.out[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    }
    return;
  }

  auto scaled = [&](int64_t i) { return __fdiv_rn(load_logit(p, logits, i), temp); };

  // ---- top-k: key of the k-th largest value ------------------------------
  const int32_t k_req = p.top_k[row];
  const bool use_k = k_req > 0 && (int64_t)k_req < V;
  uint32_t k_key = 0;          // keep key > k_key, and ties at k_key up to k_ties
  int64_t k_ties = 0;          // how many tokens equal to k_key are kept (lowest indices)
  bool k_tie_cut = false;
  if (use_k) {
    uint32_t prefix = 0, rank = (uint32_t)k_req;  // rank-th largest among keys matching prefix
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kSampleThreads) hist_count[b] = 0;
      __syncthreads();
      const uint32_t mask_hi = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int64_t i = tid; i < V; i += kSampleThreads) {
        const uint32_t key = order_key(scaled(i));
        if ((key & mask_hi) == prefix) atomicAdd(&hist_count[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t acc = 0;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + hist_count[b] >= rank) break;
          acc += hist_count[b];
        }
        sel_prefix_sh = prefix | ((uint32_t)b << shift);
        sel_rank_sh = rank - acc;
      }
      __syncthreads();
      prefix = sel_prefix_sh;
      rank = sel_rank_sh;
    }
    k_key = prefix;
    k_ties = rank;  // of the tokens equal to the k-th value, the first `rank` are kept
    k_tie_cut = true;
  }
  // Tie handling at the k cut: a token equal to k_key is kept when fewer than
  // k_ties equal tokens precede it (index order), counted per thread chunk.
  // Each thread owns a contiguous chunk of the row for the in-order passes.
  const int64_t chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int64_t c0 = min((int64_t)tid * chunk, V), c1 = min(c0 + chunk, V);
  int64_t ties_before = 0;  // equal-to-k_key tokens in earlier chunks
  if (k_tie_cut) {
    uint32_t mine = 0;
    for (int64_t i = c0; i < c1; ++i) mine += order_key(scaled(i)) == k_key;
    chunk_mass[tid] = (float)mine;  // exact for counts below 2^24
    __syncthreads();
    // Exclusive prefix over the threads (sequential per warp of sums is
    // enough here: 1024 entries).
    if (tid == 0) {
      float run = 0.f;
      for (int t = 0; t < kSampleThreads; ++t) {
        const float c = chunk_mass[t];
        chunk_mass[t] = run;
        run += c;
      }
    }
    __syncthreads();
    ties_before = (int64_t)chunk_mass[tid];
    __syncthreads();
  }
  auto kept_by_k = [&](uint32_t key, int64_t& ties_seen) -> bool {
    if (!k_tie_cut) return true;
    if (key > k_key) return true;
    if (key < k_key) return false;
    return ties_before + ties_seen++ < k_ties;
  };

  // ---- softmax statistics over the top-k set ----------------------------
  float mx = -INFINITY;
  {
    int64_t seen = 0;
    for (int64_t i = c0; i < c1; ++i) {
      const float x = scaled(i);
      if (kept_by_k(order_key(x), seen)) mx = fmaxf(mx, x);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __syncthreads();
  if (lane == 0) red_f[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red_f[0];
    for (int w = 1; w < kWarpsPerCta; ++w) m = fmaxf(m, red_f[w]);
    red_f[0] = m;
  }
  __syncthreads();
  mx = red_f[0];
  __syncthreads();
  float zsum = 0.f;
  {
    int64_t seen = 0;
    for (int64_t i = c0; i < c1; ++i) {
      const float x = scaled(i);
      if (kept_by_k(order_key(x), seen)) zsum += expf(x - mx);
    }
  }
  const float Z = block_sum(zsum, red_f);

  // ---- top-p: boundary key -----------------------------------------------
  const float top_p = p.top_p[row];
  const bool use_p = top_p < 1.f;
  uint32_t p_key = 0;       // keep key > p_key, and ties at p_key up to p_ties
  int64_t p_ties = 0;
  if (use_p) {
    // Find the smallest key b (a token's) with mass(key > b) <= top_p: digit
    // by digit from the top, the bin where the mass above first exceeds
    // top_p once the bin itself is added.
    uint32_t prefix = 0;
    float above = 0.f;  // normalised mass of keys above the current prefix range
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kSampleThreads) {
        hist_count[b] = 0;
        hist_mass[b] = 0ull;
      }
      __syncthreads();
      const uint32_t mask_hi = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      {
        int64_t seen = 0;
        for (int64_t i = c0; i < c1; ++i) {
          const float x = scaled(i);
          const uint32_t key = order_key(x);
          if (!kept_by_k(key, seen) || (key & mask_hi) != prefix) continue;
          const float q = expf(x - mx) / Z;  // in [0, 1]
          atomicAdd(&hist_mass[(key >> shift) & 255u], (unsigned long long)(q * 1099511627776.0f));
          atomicAdd(&hist_count[(key >> shift) & 255u], 1u);
        }
      }
      __syncthreads();
      if (tid == 0) {
        // The first non-empty bin from the top whose mass takes the running
        // total past top_p; when none does (everything fits), the lowest
        // non-empty bin.
        double acc = above;
        int sel = -1, last = -1;
        double acc_at_last = acc;
        for (int b = 255; b >= 0; --b) {
          if (hist_count[b] == 0) continue;
          const double m = (double)hist_mass[b] * (1.0 / 1099511627776.0);
          if (acc + m > (double)top_p) {
            sel = b;
            break;
          }
          last = b;
          acc_at_last = acc;
          acc += m;
        }
        if (sel < 0) {
          sel = last < 0 ? 0 : last;
          acc = acc_at_last;
        }
        sel_prefix_sh = prefix | ((uint32_t)sel << shift);
        sel_mass_sh = (float)acc;
      }
      __syncthreads();
      prefix = sel_prefix_sh;
      above = sel_mass_sh;
    }
    p_key = prefix;
    // Ties at the boundary value, in index order: token t of them is kept
    // while the mass before it stays <= top_p.
    const float q = expf(__uint_as_float((p_key & 0x80000000u) ? (p_key & 0x7FFFFFFFu) : ~p_key) - mx) / Z;
    p_ties = q > 0.f ? (int64_t)floorf((top_p - above) / q) + 1 : (int64_t)1;
    if (p_ties < 1) p_ties = 1;
  }
  int64_t p_ties_before = 0;
  if (use_p) {
    uint32_t mine = 0;
    int64_t seen = 0;
    for (int64_t i = c0; i < c1; ++i) {
      const uint32_t key = order_key(scaled(i));
      if (kept_by_k(key, seen) && key == p_key) ++mine;
    }
    chunk_mass[tid] = (float)mine;
    __syncthreads();
    if (tid == 0) {
      float run = 0.f;
      for (int t = 0; t < kSampleThreads; ++t) {
        const float cnt = chunk_mass[t];
        chunk_mass[t] = run;
        run += cnt;
      }
    }
    __syncthreads();
    p_ties_before = (int64_t)chunk_mass[tid];
    __syncthreads();
  }

  // ---- draw: inverse CDF over the kept tokens in index order -------------
  auto kept_mass = [&](bool accumulate_only, float target, int64_t* pick) -> float {
    float m = 0.f;
    int64_t seen_k = 0, seen_p = 0;
    for (int64_t i = c0; i < c1; ++i) {
      const float x = scaled(i);
      const uint32_t key = order_key(x);
      if (!kept_by_k(key, seen_k)) continue;
      if (use_p) {
        if (key < p_key) continue;
        if (key == p_key && p_ties_before + seen_p++ >= p_ties) continue;
      }
      m += expf(x - mx);
      *pick = i;  // the last kept index so far
      if (!accumulate_only && m > target) return m;
    }
    return m;
  };
  int64_t last_kept = -1;
  const float mine = kept_mass(true, 0.f, &last_kept);
  chunk_mass[tid] = mine;
  chunk_last[tid] = last_kept;
  __syncthreads();
  if (tid == 0) {
    float run = 0.f;
    for (int t = 0; t < kSampleThreads; ++t) {
      const float c = chunk_mass[t];
      chunk_mass[t] = run;
      run += c;
    }
    red_f[0] = run;  // total kept mass
    pick_sh = -1;
  }
  __syncthreads();
  const float total = red_f[0];
  const uint4 r = philox4x32_10(
      make_uint4((uint32_t)p.sample_index[row], (uint32_t)((uint64_t)p.sample_index[row] >> 32), 0u, 0u),
      make_uint2((uint32_t)p.seed[row], (uint32_t)(p.seed[row] >> 32)));
  const float u = (float)(r.x >> 8) * (1.0f / 16777216.0f);  // [0, 1)
  const float target = u * total;
  const float before = chunk_mass[tid];
  if (mine > 0.f && target >= before && target < before + mine) {
    int64_t pick = -1;
    kept_mass(false, target - before, &pick);
    pick_sh = pick;  // one thread's range holds the target
  }
  __syncthreads();
  if (tid == 0) {
    int64_t pick = pick_sh;
    // Rounding left the target at the very end: the last kept token.
    for (int t = kSampleThreads - 1; t >= 0 && pick < 0; --t) pick = chunk_last[t];
    p.out[row] = pick < 0 ? 0 : pick;
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
  if (a.num_rows > INT32_MAX) return MVB_ERR_UNSUPPORTED_SHAPE;
  sample_kernel<<<(unsigned)a.num_rows, kSampleThreads, 0, a.stream>>>(p);
  return check_launch();
}

}  // namespace mvb
