// Device-side token sampling: Sampler::sample (sampler.rs:47-109) with the
// reference's RNG, so non-greedy decoding needs no logits copy to the host.
//
// RNG: rand 0.8.8's StdRng = rand_chacha 0.3.1's ChaCha12Rng seeded by
// rand_core 0.6.4's seed_from_u64 (published algorithms, restated): the u64
// seed expands through PCG32 (XSH-RR, state advanced by the 64-bit LCG
// 6364136223846793005 / 11634580027462260723 before each output) into the
// eight key words; ChaCha with 12 rounds, 64-bit block counter in state
// words 12-13 and stream 0 in words 14-15; each refill makes four
// consecutive blocks (64 words) consumed in order; gen::<f32>() is
// (next_u32 >> 8) * 2^-24. The state lives in device memory and advances
// only on the device.
//
// Per draw (temperature > 0, top_k != 1; otherwise the greedy argmax):
//   samp_max_kernel    per-CTA max of logits / temperature
//   samp_exp_kernel    e = exp(l / T - max) per contiguous chunk, f64 chunk sums
//   samp_norm_kernel   p = e / sum (the softmax of tensor.rs:230-245), f64
//                      chunk sums of p
//   samp_pick_kernel   one CTA: the uniform draw and the choice
// Choice, no filters (sampler.rs:57-67): the chunk where the f64 running sum
// of p reaches r, then the reference's sequential f32 `r -= p` scan inside
// it. With top-k / top-p (sampler.rs:69-108) and at most kSampCand
// candidates: the k-th largest probability by bisection over the f32 bit
// patterns (non-negative floats order like their bits), the candidates
// gathered (ties at the boundary by lower index, as the oracle), a bitonic
// sort by (p descending, index ascending), then the reference's own f32
// steps serially: cumulative top-p cutoff, candidate total, r * total scan.
// Larger candidate sets (top_k = 0 or > kSampCand over a large vocabulary)
// locate the top-p cutoff and the draw by f64 mass bisection instead.
//
// Differences from the reference, all at rounding level: exp is the f64
// exponential rounded to f32 (the reference's f32::exp is glibc's expf,
// whose result can sit one ulp away), the softmax sum and the running sums
// that pick a chunk are f64 rather than a sequential f32 fold (over a
// 151,936-entry vocabulary that fold drops every term below half an ulp of
// its running sum, a few 1e-4 of the mass), and the large candidate path
// compares f64 masses. A draw differs from the reference's only when the
// uniform falls within that rounding of a boundary, and then lands on a
// neighbouring token.
#include <algorithm>
#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace minq {

constexpr int kSampCand = 4096;   // candidates sorted in shared memory
constexpr int kSampChunk = 4096;  // max elements per chunk of the no-filter scan
constexpr int kSampMaxGrid = 1024;
constexpr int kSampPickThreads = 1024;

struct SampRng {  // StdRng state (device)
  uint32_t key[8];
  unsigned long long block;
  uint32_t buf[64];
  uint32_t idx;
};

struct SampParams {
  const float* logits;
  size_t n;
  float temperature;
  size_t k;        // top-k survivors (n when the filter is off)
  float top_p;
  int fast;        // no filters: draw over the whole distribution
  int grid;        // chunks
  size_t chunk;    // elements per chunk (<= kSampChunk)
  float* p;        // [n] probabilities (16-byte aligned)
  float* part_max; // [grid]
  double* part_e;  // [grid]
  double* part_p;  // [grid]
  SampRng* rng;
  uint32_t* out;   // the token
};

__device__ __forceinline__ uint32_t samp_rotl(uint32_t x, int r) {
  return (x << r) | (x >> (32 - r));
}

__device__ void chacha12_block(const uint32_t* key, unsigned long long ctr, uint32_t* out) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
#pragma unroll
  for (int i = 0; i < 8; ++i) s[4 + i] = key[i];
  s[12] = (uint32_t)ctr;
  s[13] = (uint32_t)(ctr >> 32);
  s[14] = 0u;
  s[15] = 0u;
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = s[i];
#define SAMP_QR(a, b, c, d)                          \
  x[a] += x[b]; x[d] = samp_rotl(x[d] ^ x[a], 16); \
  x[c] += x[d]; x[b] = samp_rotl(x[b] ^ x[c], 12); \
  x[a] += x[b]; x[d] = samp_rotl(x[d] ^ x[a], 8);  \
  x[c] += x[d]; x[b] = samp_rotl(x[b] ^ x[c], 7);
#pragma unroll
  for (int r = 0; r < 12; r += 2) {
    SAMP_QR(0, 4, 8, 12) SAMP_QR(1, 5, 9, 13) SAMP_QR(2, 6, 10, 14) SAMP_QR(3, 7, 11, 15)
    SAMP_QR(0, 5, 10, 15) SAMP_QR(1, 6, 11, 12) SAMP_QR(2, 7, 8, 13) SAMP_QR(3, 4, 9, 14)
  }
#undef SAMP_QR
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

// RngCore::next_u32 of the block RNG (one thread).
__device__ uint32_t samp_next_u32(SampRng* g) {
  if (g->idx >= 64) {
    for (int b = 0; b < 4; ++b) chacha12_block(g->key, g->block + b, g->buf + 16 * b);
    g->block += 4;
    g->idx = 0;
  }
  return g->buf[g->idx++];
}

__device__ __forceinline__ double samp_warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block sum of a double over blockDim.x threads (a multiple of 32, <= 1024);
// every thread gets the same result (an xor butterfly leaves every lane with
// bit-identical sums).
__device__ double samp_block_sum(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = samp_warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.0;
  return samp_warp_sum(v);
}

__device__ float samp_block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : -INFINITY;
  return warp_max(v);
}

// --- softmax over the grid ---------------------------------------------------

__global__ void __launch_bounds__(256) samp_max_kernel(SampParams q) {
  __shared__ float red[32];
  pdl_wait();
  float m = -INFINITY;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q.n;
       i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, q.logits[i] / q.temperature);
  m = samp_block_max(m, red);
  if (threadIdx.x == 0) q.part_max[blockIdx.x] = m;
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(256) samp_exp_kernel(SampParams q) {
  __shared__ float redf[32];
  __shared__ double redd[32];
  pdl_wait();
  float m = -INFINITY;
  for (int b = threadIdx.x; b < q.grid; b += blockDim.x) m = fmaxf(m, q.part_max[b]);
  m = samp_block_max(m, redf);
  const size_t lo = blockIdx.x * q.chunk, hi = min(q.n, lo + q.chunk);
  double s = 0.0;
  for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float d = q.logits[i] / q.temperature - m;
    const float e = (float)exp((double)d);
    q.p[i] = e;
    s += (double)e;
  }
  s = samp_block_sum(s, redd);
  if (threadIdx.x == 0) q.part_e[blockIdx.x] = s;
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(256) samp_norm_kernel(SampParams q) {
  __shared__ double redd[32];
  pdl_wait();
  double t = 0.0;
  for (int b = threadIdx.x; b < q.grid; b += blockDim.x) t += q.part_e[b];
  const float sum = (float)samp_block_sum(t, redd);
  const size_t lo = blockIdx.x * q.chunk, hi = min(q.n, lo + q.chunk);
  double s = 0.0;
  for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float v = q.p[i];
    if (sum > 0.0f) v = v / sum;  // tensor.rs:240-244: divide only when the sum is positive
    q.p[i] = v;
    s += (double)v;
  }
  s = samp_block_sum(s, redd);
  if (threadIdx.x == 0) q.part_p[blockIdx.x] = s;
  pdl_launch_dependents();
}

// --- the choice (one CTA) ----------------------------------------------------

constexpr uint32_t kAllTies = 0xFFFFFFFFu;

struct SampShared {
  unsigned long long cand[kSampCand];  // (key << 32) | ~index; the no-filter scan stages floats here
  double redd[32];
  uint32_t wcnt[32];
  uint32_t count;
  uint32_t result;
  int found;
  float u;
  float rr;
};

__device__ __forceinline__ uint32_t samp_key(const float* p, size_t i) {
  return __float_as_uint(p[i]);
}

// Count (and, with MASS, f64 mass) of {i : key_i >= x} over the whole
// vector (every thread gets them). p is 16-byte aligned: float4 loads,
// several in flight per thread.
template <bool MASS>
__device__ void samp_measure_t(const float* p, size_t n, uint32_t x, SampShared& sh, double& cnt,
                               double& mass) {
  uint32_t c = 0;
  double m = 0.0;
  const size_t n4 = n / 4;
  const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll 4
  for (size_t j = threadIdx.x; j < n4; j += blockDim.x) {
    const float4 v = p4[j];
    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const bool in = __float_as_uint(e[q]) >= x;
      c += in ? 1u : 0u;
      if (MASS) m += in ? (double)e[q] : 0.0;
    }
  }
  for (size_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t k = samp_key(p, i);
    if (k >= x) {
      c += 1u;
      if (MASS) m += (double)__uint_as_float(k);
    }
  }
  cnt = samp_block_sum((double)c, sh.redd);
  mass = MASS ? samp_block_sum(m, sh.redd) : 0.0;
}

__device__ __forceinline__ void samp_measure(const float* p, size_t n, uint32_t x, bool with_mass,
                                             SampShared& sh, double& cnt, double& mass) {
  if (with_mass)
    samp_measure_t<true>(p, n, x, sh, cnt, mass);
  else
    samp_measure_t<false>(p, n, x, sh, cnt, mass);
}

// A candidate set S = {key > lo_key} plus the first lo_ties elements (index
// order) with key == lo_key (all of them for kAllTies). samp_walk() finds the
// rank where S, taken in the order (key descending, index ascending), first
// reaches `target` elements (by_mass = false) or probability mass (true):
// tau = that element's key, t = its 1-based position among the ties at tau
// in S, above = count / mass of S with key > tau. Bisection over the keys
// (at most 31 passes over the vector). S must not be empty.
struct SampWalk {
  uint32_t tau;
  uint32_t t;
  double above_cnt, above_mass;
};

__device__ SampWalk samp_walk(const float* p, size_t n, uint32_t lo_key, uint32_t lo_ties,
                              bool by_mass, double target, SampShared& sh) {
  double clo, mlo, c1, m1;
  samp_measure(p, n, lo_key, by_mass, sh, clo, mlo);
  if (lo_ties != kAllTies) {  // cap the ties at lo_key
    samp_measure(p, n, lo_key + 1, by_mass, sh, c1, m1);
    const double take = fmin(clo - c1, (double)lo_ties);
    clo = c1 + take;
    mlo = m1 + take * (double)__uint_as_float(lo_key);
  }
  // a target beyond S (rounding) means its last element; a zero mass
  // target its first (the reference's scan stops at the first r <= 0)
  target = fmin(target, by_mass ? mlo : clo);
  if (by_mass) target = fmax(target, 1e-300);
  uint32_t lo = lo_key, hi = 0x7F800001u;  // F(hi) = 0: above every finite key
  double chi = 0.0, mhi = 0.0;
  while (hi - lo > 1) {  // invariant: F(lo) >= target > F(hi)
    const uint32_t mid = lo + (hi - lo) / 2;
    double c, m;
    samp_measure(p, n, mid, by_mass, sh, c, m);
    if ((by_mass ? m : c) >= target) {
      lo = mid;
      clo = c;
      mlo = m;
    } else {
      hi = mid;
      chi = c;
      mhi = m;
    }
  }
  SampWalk w;
  w.tau = lo;
  w.above_cnt = chi;
  w.above_mass = mhi;
  const double avail = clo - chi;  // ties at tau that belong to S
  double t;
  if (by_mass) {
    const double pv = (double)__uint_as_float(lo);
    t = pv > 0.0 ? ceil((target - mhi) / pv) : avail;
  } else {
    t = target - chi;
  }
  t = fmax(1.0, fmin(t, avail));
  w.t = (uint32_t)t;
  return w;
}

// Ordered pass over the vector in tiles of 4 * blockDim.x elements (four
// consecutive ones per thread): every element whose key is above tau, or
// that is one of the first `ties` elements with key == tau (index order), is
// visited as visit(i, key, rank), rank = its 0-based position among the ties.
template <class Visit>
__device__ void samp_ordered(const float* p, size_t n, uint32_t tau, uint32_t ties,
                             SampShared& sh, Visit visit) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t base = 0;
  for (size_t t0 = 0; t0 < n; t0 += 4 * (size_t)blockDim.x) {
    const size_t i0 = t0 + 4 * (size_t)threadIdx.x;
    uint32_t key[4];
    if (i0 + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(p + i0);
      key[0] = __float_as_uint(v.x);
      key[1] = __float_as_uint(v.y);
      key[2] = __float_as_uint(v.z);
      key[3] = __float_as_uint(v.w);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) key[q] = i0 + q < n ? samp_key(p, i0 + q) : 0u;
    }
    uint32_t mine = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) mine += (i0 + q < n && key[q] == tau) ? 1u : 0u;
    uint32_t incl = mine;  // inclusive warp scan of the ties
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) sh.wcnt[warp] = incl;
    __syncthreads();
    uint32_t wbase = 0, total = 0;
    for (int w = 0; w < nw; ++w) {
      const uint32_t c = sh.wcnt[w];
      wbase += w < warp ? c : 0u;
      total += c;
    }
    uint32_t rank = base + wbase + incl - mine;  // this thread's first tie
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const size_t i = i0 + q;
      if (i >= n) break;
      const bool tie = key[q] == tau;
      if (key[q] > tau || (tie && (ties == kAllTies || rank < ties))) visit(i, key[q], rank);
      if (tie) ++rank;
    }
    base += total;
    __syncthreads();  // wcnt is rewritten by the next tile
  }
}

// Candidates (key > tau, or among the first `ties` at tau) into sh.cand,
// sorted by (key descending, index ascending); returns their number.
__device__ uint32_t samp_gather_sorted(const float* p, size_t n, uint32_t tau, uint32_t ties,
                                       SampShared& sh) {
  if (threadIdx.x == 0) sh.count = 0;
  __syncthreads();
  samp_ordered(p, n, tau, ties, sh, [&](size_t i, uint32_t key, uint32_t) {
    const uint32_t slot = atomicAdd(&sh.count, 1u);
    if (slot < (uint32_t)kSampCand)
      sh.cand[slot] = ((unsigned long long)key << 32) | (uint32_t)~(uint32_t)i;
  });
  __syncthreads();
  const uint32_t m = min(sh.count, (uint32_t)kSampCand);
  uint32_t N = 2;
  while (N < m) N <<= 1;
  for (uint32_t i = m + threadIdx.x; i < N; i += blockDim.x) sh.cand[i] = 0ull;  // rank last
  __syncthreads();
  for (uint32_t k = 2; k <= N; k <<= 1)
    for (uint32_t j = k >> 1; j > 0; j >>= 1) {
      for (uint32_t i = threadIdx.x; i < N; i += blockDim.x) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = sh.cand[i], b = sh.cand[ixj];
          const bool desc = (i & k) == 0;  // this half sorts descending
          if (desc ? a < b : a > b) {
            sh.cand[i] = b;
            sh.cand[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  return m;
}

// sampler.rs:84-108 on m sorted candidates, by one thread: the top-p cutoff
// by the f32 cumulative sum in rank order, the f32 total of the kept ones,
// then r = u * total and the `r -= p` scan.
__device__ uint32_t samp_pick_sorted(const SampShared& sh, uint32_t m, float top_p, float u) {
  if (m == 0) return 0u;
  uint32_t cutoff = m;
  float cum = 0.0f;
  for (uint32_t r = 0; r < m; ++r) {
    cum += __uint_as_float((uint32_t)(sh.cand[r] >> 32));
    if (cum >= top_p) {
      cutoff = r + 1;
      break;
    }
  }
  float total = 0.0f;
  for (uint32_t r = 0; r < cutoff; ++r) total += __uint_as_float((uint32_t)(sh.cand[r] >> 32));
  float rr = u * total;
  for (uint32_t r = 0; r < cutoff; ++r) {
    rr -= __uint_as_float((uint32_t)(sh.cand[r] >> 32));
    if (rr <= 0.0f) return ~(uint32_t)sh.cand[r];
  }
  return ~(uint32_t)sh.cand[cutoff - 1];
}

// Mass of the set S (see samp_walk).
__device__ double samp_set_mass(const float* p, size_t n, uint32_t lo_key, uint32_t lo_ties,
                                SampShared& sh) {
  double c, m;
  samp_measure(p, n, lo_key, true, sh, c, m);
  if (lo_ties == kAllTies) return m;
  double c1, m1;
  samp_measure(p, n, lo_key + 1, true, sh, c1, m1);
  return m1 + fmin(c - c1, (double)lo_ties) * (double)__uint_as_float(lo_key);
}

// Index of the t-th (1-based) element with key == tau in index order, or
// `fallback` when there is none (every thread gets it).
__device__ uint32_t samp_nth_tie(const float* p, size_t n, uint32_t tau, uint32_t t,
                                 uint32_t fallback, SampShared& sh) {
  if (threadIdx.x == 0) sh.result = fallback;
  __syncthreads();
  samp_ordered(p, n, tau, t, sh, [&](size_t i, uint32_t key, uint32_t rank) {
    if (key == tau && rank + 1 == t) sh.result = (uint32_t)i;
  });
  __syncthreads();
  return sh.result;
}

// sampler.rs:57-67: r -= p[i] in index order until r <= 0, else the last
// index. The f64 chunk sums pick the chunk where r runs out; thread 0 runs
// the f32 scan from there (into later chunks if rounding carries it on).
__device__ uint32_t samp_fast(const SampParams& q, float u, SampShared& sh) {
  if (threadIdx.x == 0) {
    double acc = 0.0;
    int b = 0;
    for (; b < q.grid - 1; ++b) {
      if (acc + q.part_p[b] >= (double)u) break;
      acc += q.part_p[b];
    }
    sh.count = (uint32_t)b;
    sh.rr = (float)((double)u - acc);
    sh.found = 0;
    sh.result = (uint32_t)(q.n - 1);
  }
  __syncthreads();
  const uint32_t b0 = sh.count;
  float* buf = reinterpret_cast<float*>(sh.cand);  // chunk <= kSampChunk floats
  for (uint32_t b = b0; b < (uint32_t)q.grid; ++b) {
    const size_t lo = (size_t)b * q.chunk, hi = min(q.n, lo + q.chunk);
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) buf[i - lo] = q.p[i];
    __syncthreads();
    if (threadIdx.x == 0) {
      float rr = sh.rr;
      for (size_t i = lo; i < hi; ++i) {
        rr -= buf[i - lo];
        if (rr <= 0.0f) {
          sh.result = (uint32_t)i;
          sh.found = 1;
          break;
        }
      }
      sh.rr = rr;
    }
    __syncthreads();
    if (sh.found) break;
  }
  return sh.result;
}

__global__ void __launch_bounds__(kSampPickThreads) samp_pick_kernel(SampParams q) {
  __shared__ SampShared sh;
  pdl_wait();
  if (threadIdx.x == 0) {
    const uint32_t x = samp_next_u32(q.rng);
    sh.u = (float)(x >> 8) * (1.0f / 16777216.0f);  // rand's Standard f32
  }
  __syncthreads();
  const float u = sh.u;
  uint32_t token;
  if (q.fast) {
    token = samp_fast(q, u, sh);
  } else {
    // the top-k survivors A: keys above tau_a plus the first ties_a at tau_a
    uint32_t tau_a = 0u, ties_a = kAllTies;
    size_t m_a = q.n;
    if (q.k < q.n) {
      const SampWalk w = samp_walk(q.p, q.n, 0u, kAllTies, false, (double)q.k, sh);
      tau_a = w.tau;
      ties_a = w.t;
      m_a = q.k;
    }
    bool done = false;
    if (m_a <= (size_t)kSampCand) {
      const uint32_t m = samp_gather_sorted(q.p, q.n, tau_a, ties_a, sh);
      if (threadIdx.x == 0) sh.result = samp_pick_sorted(sh, m, q.top_p, u);
      __syncthreads();
      token = sh.result;
      done = true;
    } else if (q.top_p < 1.0f) {
      // a rank prefix a little past the top-p mass; when it is small the
      // reference's f32 steps run on it exactly
      const SampWalk w = samp_walk(q.p, q.n, tau_a, ties_a, true, (double)q.top_p + 1e-3, sh);
      if (w.above_cnt + (double)w.t <= (double)kSampCand) {
        const uint32_t m = samp_gather_sorted(q.p, q.n, w.tau, w.t, sh);
        if (threadIdx.x == 0) sh.result = samp_pick_sorted(sh, m, q.top_p, u);
        __syncthreads();
        token = sh.result;
        done = true;
      }
    }
    if (!done) {  // large candidate set: cutoff and draw by f64 mass
      uint32_t tau_p = tau_a, ties_p = ties_a;
      double total;
      if (q.top_p < 1.0f) {
        const SampWalk w = samp_walk(q.p, q.n, tau_a, ties_a, true, (double)q.top_p, sh);
        tau_p = w.tau;
        ties_p = w.t;
        total = w.above_mass + (double)w.t * (double)__uint_as_float(w.tau);
      } else {
        total = samp_set_mass(q.p, q.n, tau_a, ties_a, sh);
      }
      const SampWalk d = samp_walk(q.p, q.n, tau_p, ties_p, true, (double)u * total, sh);
      token = samp_nth_tie(q.p, q.n, d.tau, d.t, (uint32_t)(q.n - 1), sh);
    }
  }
  if (threadIdx.x == 0) *q.out = token;
  pdl_launch_dependents();
}

__global__ void samp_raw_kernel(SampRng* g, size_t n, uint32_t* out) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0)
    for (size_t i = 0; i < n; ++i) out[i] = samp_next_u32(g);
}

}  // namespace minq

// ---------------------------------------------------------------------------
// C ABI

struct minq_sampler {
  float temperature = 0.0f;
  size_t top_k = 0;
  float top_p = 1.0f;
  int device = 0;
  minq::SampRng* rng = nullptr;
  float* p = nullptr;  // [cap] probabilities
  size_t cap = 0;
  float* part_max = nullptr;  // [kSampMaxGrid]
  double* part_e = nullptr;
  double* part_p = nullptr;
  unsigned long long* arg = nullptr;  // greedy argmax scratch
  float* staged = nullptr;            // host logits of minq_sampler_sample
  size_t staged_cap = 0;
  uint32_t* tok = nullptr;
  uint32_t* raw = nullptr;
  size_t raw_cap = 0;
};

int minq::sampler_device(const minq_sampler* s) { return s ? s->device : -1; }

namespace {

using namespace minq;

minq_status grow(void** ptr, size_t* cap, size_t need, size_t elem) {
  if (*cap >= need) return MINQ_OK;
  cudaFree(*ptr);
  *ptr = nullptr;
  *cap = 0;
  MINQ_CUDA_TRY(cudaMalloc(ptr, need * elem));
  *cap = need;
  return MINQ_OK;
}

}  // namespace

extern "C" {

minq_status minq_sampler_new(float temperature, size_t top_k, float top_p, uint64_t seed,
                             minq_sampler** out) {
  if (!out) return fail(MINQ_ERR_ARG, "null argument");
  *out = nullptr;
  minq_sampler* s = new minq_sampler();
  s->temperature = temperature;
  s->top_k = top_k;
  s->top_p = top_p;
  cudaGetDevice(&s->device);
  SampRng g{};
  uint64_t st = seed;  // seed_from_u64: PCG32 outputs as the key words
  for (int i = 0; i < 8; ++i) {
    st = st * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xs = (uint32_t)(((st >> 18) ^ st) >> 27);
    const unsigned rot = (unsigned)(st >> 59);
    g.key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  g.block = 0;
  g.idx = 64;  // empty buffer: the first draw refills
  cudaError_t e = cudaMalloc(&s->rng, sizeof(SampRng));
  if (e == cudaSuccess) e = cudaMemcpy(s->rng, &g, sizeof(SampRng), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&s->part_max, kSampMaxGrid * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&s->part_e, kSampMaxGrid * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&s->part_p, kSampMaxGrid * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&s->arg, 32 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&s->tok, 16);
  if (e != cudaSuccess) {
    minq_sampler_free(s);
    return cuda_fail(e, "cudaMalloc(sampler)");
  }
  *out = s;
  return MINQ_OK;
}

void minq_sampler_free(minq_sampler* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  cudaDeviceSynchronize();
  for (void* b : {(void*)s->rng, (void*)s->p, (void*)s->part_max, (void*)s->part_e,
                  (void*)s->part_p, (void*)s->arg, (void*)s->staged, (void*)s->tok,
                  (void*)s->raw})
    cudaFree(b);
  delete s;
}

minq_status minq_sampler_sample_device(minq_sampler* s, const float* d_logits, size_t n,
                                       uint32_t* d_token, void* stream) {
  if (!s || !d_token || (n && !d_logits)) return fail(MINQ_ERR_ARG, "null argument");
  MINQ_CUDA_TRY(cudaSetDevice(s->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {  // sampler.rs:48-50
    MINQ_CUDA_TRY(cudaMemsetAsync(d_token, 0, 4, st));
    return MINQ_OK;
  }
  if (n > (size_t)kSampMaxGrid * kSampChunk)
    return fail(MINQ_ERR_ARG, "device sampling takes at most 4194304 logits");
  if (s->temperature <= 0.0f || s->top_k == 1)  // sampler.rs:51-53
    return launch_argmax_rows(d_logits, n, 1, d_token, s->arg, st);
  MINQ_TRY(grow(reinterpret_cast<void**>(&s->p), &s->cap, n, sizeof(float)));
  SampParams q{};
  q.logits = d_logits;
  q.n = n;
  q.temperature = s->temperature;
  q.k = s->top_k == 0 ? n : std::min(s->top_k, n);
  q.top_p = s->top_p;
  q.fast = (s->top_k == 0 || s->top_k >= n) && s->top_p >= 1.0f;
  const size_t need = (n + kSampChunk - 1) / kSampChunk;
  const size_t want = std::min<size_t>((size_t)sm_count(), (n + 255) / 256);
  q.grid = (int)std::max<size_t>(1, std::max(need, want));
  q.chunk = (n + q.grid - 1) / q.grid;
  q.p = s->p;
  q.part_max = s->part_max;
  q.part_e = s->part_e;
  q.part_p = s->part_p;
  q.rng = s->rng;
  q.out = d_token;
  MINQ_CUDA_TRY(launch_k(samp_max_kernel, dim3(q.grid), dim3(256), 0, st, q));
  MINQ_CUDA_TRY(launch_k(samp_exp_kernel, dim3(q.grid), dim3(256), 0, st, q));
  MINQ_CUDA_TRY(launch_k(samp_norm_kernel, dim3(q.grid), dim3(256), 0, st, q));
  MINQ_CUDA_TRY(launch_k(samp_pick_kernel, dim3(1), dim3(kSampPickThreads), 0, st, q));
  return MINQ_OK;
}

minq_status minq_sampler_sample(minq_sampler* s, const float* logits, size_t n,
                                uint32_t* token_out) {
  if (!s || !token_out || (n && !logits)) return fail(MINQ_ERR_ARG, "null argument");
  MINQ_CUDA_TRY(cudaSetDevice(s->device));
  MINQ_TRY(grow(reinterpret_cast<void**>(&s->staged), &s->staged_cap, std::max<size_t>(n, 1),
                sizeof(float)));
  if (n) MINQ_CUDA_TRY(cudaMemcpy(s->staged, logits, n * 4, cudaMemcpyHostToDevice));
  MINQ_TRY(minq_sampler_sample_device(s, s->staged, n, s->tok, nullptr));
  MINQ_CUDA_TRY(cudaMemcpy(token_out, s->tok, 4, cudaMemcpyDeviceToHost));
  return take_device_status();
}

minq_status minq_sampler_rng_u32(minq_sampler* s, size_t n, uint32_t* out) {
  if (!s || (n && !out)) return fail(MINQ_ERR_ARG, "null argument");
  if (n > (1u << 20)) return fail(MINQ_ERR_ARG, "at most 2^20 words per call");
  if (n == 0) return MINQ_OK;
  MINQ_CUDA_TRY(cudaSetDevice(s->device));
  MINQ_TRY(grow(reinterpret_cast<void**>(&s->raw), &s->raw_cap, n, sizeof(uint32_t)));
  MINQ_CUDA_TRY(launch_k(samp_raw_kernel, dim3(1), dim3(32), 0, nullptr, s->rng, n, s->raw));
  MINQ_CUDA_TRY(cudaMemcpy(out, s->raw, n * 4, cudaMemcpyDeviceToHost));
  return MINQ_OK;
}

}  // extern "C"
