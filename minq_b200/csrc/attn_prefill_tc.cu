// Causal attention of a prompt chunk on the 5th-generation tensor cores
// (flash-prefill): T consecutive query tokens at positions p0 .. p0 + T - 1
// against the head-major f32 K/V cache, whose positions 0 .. p0 + T - 1
// already hold the chunk's own keys and values. Token t of the chunk attends
// over positions 0 ..= p0 + t, exactly the reference's per-token
// attend(q, layer_cache, pos + 1) of its prompt loop (model.rs:223-248 called
// from model.rs:259-268 / 295): scores q.k * 1/sqrt(head_dim), softmax over
// the history, weighted sum of V.
//
// Work split. For a kv head the query rows are (token t, group head g) in
// the order r = t * G + g; CTA (split, m tile, kv head) takes 128 rows and
// the split's share of the 64-position key tiles the rows need (causal:
// tiles past p0 + t_last are never loaded). With several splits their
// partials (O unnormalised, running max m, sum l per row) go to a workspace
// and fp_combine_kernel merges them; with one split the CTA writes O / l.
//
// Per key tile, in one CTA of 256 threads:
//   * all threads load the tile's K and V rows from global memory (the
//     next tile's loads are issued before the current tile's MMAs are
//     waited for), split every value into tf32 hi = x with the low 13
//     mantissa bits cleared and lo = x - hi (exact), and store K hi / lo and
//     the transpose of V hi / lo into 128-byte-swizzled K-major tiles;
//   * one thread issues S = Q K^T as tcgen05.mma kind::tf32 with the query
//     rows (hi / lo, written once per CTA) as the A operand in tensor memory:
//     S = Qh Kh + Qh Kl + Ql Kh, f32 accumulation in TMEM (the dropped Ql Kl
//     term is below 2^-21 of |q||k|), so the scores carry about the f32
//     arithmetic of the reference's dot product;
//   * warps 0-3 (thread = query row = TMEM lane) read S with tcgen05.ld,
//     scale and mask it, update the running max and sum (online softmax),
//     and write P split the same way into a swizzled tile; all warps rescale
//     the O accumulator rows in TMEM when the max moved;
//   * one thread issues O += Ph Vh + Ph Vl + Pl Vh (A = P from shared memory).
// Every wait on an MMA completion is bounded (1 s, then the device status
// word and an abort that ends the CTA's loop).
#include <cuda.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "ktimer.h"
#include "pipeline.cuh"

namespace minq {

namespace {

constexpr int kFpRows = 128;    // query rows per CTA (MMA M)
constexpr int kFpKeys = 64;     // key positions per tile (S tile N, P.V K)
constexpr int kFpThreads = 256;

template <int HD>
struct FpGeom {
  // TMEM columns: Q hi | Q lo | S | O
  static constexpr int QH = 0, QL = HD, SC = 2 * HD, OC = 2 * HD + kFpKeys;
  static constexpr int TMEM_COLS = 3 * HD + kFpKeys <= 256 ? 256 : 512;
  // shared-memory tiles (1024-byte aligned), 128-byte swizzled K-major
  static constexpr int KT = kFpKeys * HD * 4;  // K hi or lo: 64 rows x HD
  static constexpr int VT = HD * kFpKeys * 4;  // V^T hi or lo: HD rows x 64
  static constexpr int PT = kFpRows * kFpKeys * 4;
  static constexpr int KH = 0, KL = KT, VH = 2 * KT, VL = 2 * KT + VT, PH = 2 * KT + 2 * VT,
                       PL = PH + PT, CTL = PL + PT;
  static constexpr size_t smem = 1024 + (size_t)CTL + 2048;
};

struct FpParams {
  const float* q;    // [T][nh][hd]
  const float* kc;   // layer cache: kv head h at kc + h * head_stride, [max_seq][hd]
  const float* vc;
  size_t head_stride;
  float* out;        // [T][nh][hd]
  float* ws;         // NS > 1: [NS][nkv][MT][128][hd + 2]
  int p0, T, nh, nkv, G, MT, NS, nkt;
  float scale;
  int* status;
};

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Descriptor of a K-major tile in the 128-byte swizzle layout (8-row groups
// 1024 bytes apart, version 1, SWIZZLE_128B); the start may sit 32 / 64 / 96
// bytes into a swizzle row to select a k step of 8 tf32 values.
__device__ __forceinline__ uint64_t sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Byte offset of float (r, k) in an R-row K-major swizzled tile: 32-float
// column groups of R x 128 bytes, 16-byte chunk c of row r at c ^ (r mod 8).
__device__ __forceinline__ uint32_t sw_off(int r, int k, int R) {
  const int kk = k & 31;
  return (uint32_t)((k >> 5) * R * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    ((((kk >> 2) ^ (r & 7))) << 4) + ((kk & 3) << 2));
}

// kind::tf32 instruction descriptor: D f32, A and B tf32, K-major, M = 128.
__device__ __forceinline__ constexpr uint32_t fp_idesc(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit words (this warp's lane quarter).
__device__ __forceinline__ void tm_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Wait for this thread's TMEM loads; the values pass through the asm so no
// use of them is scheduled before the wait.
__device__ __forceinline__ void tm_wait_ld(float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void tm_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tm_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void sts4(uint32_t a, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void sts1(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// tf32 split: hi keeps the 10 explicit mantissa bits tf32 holds (an exact
// tf32 value whichever way the tensor core converts), lo = x - hi exactly.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Bounded wait on an MMA-completion barrier: false after 1 s (status word
// and the CTA's abort flag set) or once another thread aborted.
__device__ bool fp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      if (status) atomicOr(status, kDeviceTimeout);
      return false;
    }
  }
}

template <int HD>
struct FpTile {
  static constexpr int KU = HD / 16;  // float4 of K per thread
  static constexpr int VU = HD / 32;  // 8-float pieces of V per thread
  float4 k[KU];
  float4 v[2 * VU];
};

// Global loads of key tile kt (positions >= npos read as zero): K as float4
// rows (consecutive threads, consecutive float4 of a row), V as 8-float
// pieces with the warp's lanes on 32 consecutive positions.
template <int HD>
__device__ __forceinline__ void fp_load(const FpParams& p, const float* kh_base,
                                        const float* vh_base, int kt, int npos, FpTile<HD>& t) {
  const int tid = threadIdx.x;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < FpTile<HD>::KU; ++i) {
    const int u = tid + kFpThreads * i, pos = u / (HD / 4), c4 = u % (HD / 4);
    const int gp = kt * kFpKeys + pos;
    t.k[i] = gp < npos ? __ldg(reinterpret_cast<const float4*>(kh_base + (size_t)gp * HD) + c4) : z;
  }
#pragma unroll
  for (int i = 0; i < FpTile<HD>::VU; ++i) {
    const int u = tid + kFpThreads * i, pos = u % kFpKeys, c8 = u / kFpKeys;
    const int gp = kt * kFpKeys + pos;
    const float4* src = reinterpret_cast<const float4*>(vh_base + (size_t)gp * HD + 8 * c8);
    t.v[2 * i] = gp < npos ? __ldg(src) : z;
    t.v[2 * i + 1] = gp < npos ? __ldg(src + 1) : z;
  }
}

// Split and store a loaded tile: K hi / lo as 64-row tiles, V^T hi / lo as
// HD-row tiles (k = position).
template <int HD>
__device__ __forceinline__ void fp_store(uint32_t base, const FpTile<HD>& t) {
  using G = FpGeom<HD>;
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < FpTile<HD>::KU; ++i) {
    const int u = tid + kFpThreads * i, pos = u / (HD / 4), c4 = u % (HD / 4);
    const float4 x = t.k[i];
    const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
    const float4 l = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    const uint32_t o = sw_off(pos, 4 * c4, kFpKeys);
    sts4(base + G::KH + o, h);
    sts4(base + G::KL + o, l);
  }
#pragma unroll
  for (int i = 0; i < FpTile<HD>::VU; ++i) {
    const int u = tid + kFpThreads * i, pos = u % kFpKeys, c8 = u / kFpKeys;
    const float vv[8] = {t.v[2 * i].x,     t.v[2 * i].y,     t.v[2 * i].z,     t.v[2 * i].w,
                         t.v[2 * i + 1].x, t.v[2 * i + 1].y, t.v[2 * i + 1].z, t.v[2 * i + 1].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float h = tf32_hi(vv[e]);
      const uint32_t o = sw_off(8 * c8 + e, pos, HD);
      sts1(base + G::VH + o, h);
      sts1(base + G::VL + o, vv[e] - h);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(kFpThreads, 1) fp_attn_kernel(const __grid_constant__ FpParams p) {
  using G = FpGeom<HD>;
  extern __shared__ unsigned char fp_sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t base = (smem_u32(fp_sm) + 1023u) & ~1023u;
  unsigned char* gb = fp_sm + (base - smem_u32(fp_sm));
  float* corr = reinterpret_cast<float*>(gb + G::CTL);  // [128] rescale of O per row
  float* rowm = corr + kFpRows;
  float* rowl = rowm + kFpRows;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(rowl + kFpRows);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_o + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int split = blockIdx.x, mt = blockIdx.y, kh = blockIdx.z;
  const int Gq = p.G;
  const int t_last = min(p.T - 1, (mt * kFpRows + kFpRows - 1) / Gq);
  const int nkt_m = (p.p0 + t_last + 1 + kFpKeys - 1) / kFpKeys;  // key tiles these rows see
  const int kt0 = (int)((long long)p.nkt * split / p.NS);
  const int kt1 = min((int)((long long)p.nkt * (split + 1) / p.NS), nkt_m);
  const int ntile = max(0, kt1 - kt0);
  const int npos = p.p0 + p.T;  // positions in the cache

  if (warp == 0) {
    if (lane == 0) {
      mbar_init(bar_s, 1);
      mbar_init(bar_o, 1);
      *abort = 0;
      mbar_fence_init();
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(G::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tlane = tmem + ((uint32_t)(32 * quarter) << 16);
  pdl_wait();
  pdl_launch_dependents();

  // this thread's query row (TMEM lane 32 * quarter + lane)
  const int row = 32 * quarter + lane;
  const int rg = mt * kFpRows + row, tq = rg / Gq, gq = rg - tq * Gq;
  const bool valid = tq < p.T;
  const int lim = valid ? p.p0 + tq : -1;  // last visible key position
  const float* kbase = p.kc + (size_t)kh * p.head_stride;
  const float* vbase = p.vc + (size_t)kh * p.head_stride;

  FpTile<HD> tl;
  if (ntile > 0) fp_load<HD>(p, kbase, vbase, kt0, npos, tl);

  // query row -> TMEM as tf32 hi / lo (warps 0-3: columns [0, HD/2), 4-7 the rest)
  {
    const float* qr = p.q + ((size_t)tq * p.nh + (size_t)kh * Gq + gq) * HD + half * (HD / 2);
#pragma unroll
    for (int c = 0; c < HD / 2; c += 32) {
      float hi[32], lo[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 x = valid ? __ldg(reinterpret_cast<const float4*>(qr + c) + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[4 * i + e] = tf32_hi(xs[e]);
          lo[4 * i + e] = xs[e] - hi[4 * i + e];
        }
      }
      tm_st32(tlane + (uint32_t)(G::QH + half * (HD / 2) + c), hi);
      tm_st32(tlane + (uint32_t)(G::QL + half * (HD / 2) + c), lo);
    }
    tm_wait_st();
  }
  fence_before();
  __syncthreads();

  float m = -INFINITY, l = 0.0f;
  bool ok = true;
  for (int it = 0; it < ntile && ok; ++it) {
    const int kt = kt0 + it;
    fp_store<HD>(base, tl);
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {  // S = Qh Kh + Qh Kl + Ql Kh
      fence_after();
      constexpr uint32_t idS = fp_idesc(kFpKeys);
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        const uint32_t bo = (uint32_t)((j >> 2) * kFpKeys * 128 + (j & 3) * 32);
        const uint64_t bh = sw128(base + G::KH + bo), bl = sw128(base + G::KL + bo);
        mma_ts(tmem + G::SC, tmem + G::QH + 8 * j, bh, idS, j > 0 ? 1u : 0u);
        mma_ts(tmem + G::SC, tmem + G::QH + 8 * j, bl, idS, 1u);
        mma_ts(tmem + G::SC, tmem + G::QL + 8 * j, bh, idS, 1u);
      }
      mma_commit(bar_s);
    }
    if (it + 1 < ntile) fp_load<HD>(p, kbase, vbase, kt + 1, npos, tl);
    ok = __syncthreads_and(fp_wait(bar_s, (uint32_t)(it & 1), abort, p.status)) != 0;
    if (!ok) break;
    fence_after();
    if (warp < 4) {
      float s[2 * 32];
      tm_ld32(tlane + G::SC, s);
      tm_ld32(tlane + G::SC + 32, s + 32);
      tm_wait_ld(s);
      tm_wait_ld(s + 32);
      const int k0 = kt * kFpKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kFpKeys; ++j) {
        s[j] = k0 + j <= lim ? s[j] * p.scale : -INFINITY;
        mx = fmaxf(mx, s[j]);
      }
      const float mn = fmaxf(m, mx);
      float c = 1.0f, sum = 0.0f;
      if (mn == -INFINITY) {  // nothing visible yet (or a padding row)
#pragma unroll
        for (int j = 0; j < kFpKeys; ++j) s[j] = 0.0f;
      } else {
        c = m == -INFINITY ? 0.0f : expf(m - mn);
#pragma unroll
        for (int j = 0; j < kFpKeys; ++j) {
          s[j] = expf(s[j] - mn);  // exp(-inf) = 0 for masked keys
          sum += s[j];
        }
        m = mn;
      }
      l = l * c + sum;
      corr[row] = c;
#pragma unroll
      for (int j = 0; j < kFpKeys; j += 4) {
        const float4 h = make_float4(tf32_hi(s[j]), tf32_hi(s[j + 1]), tf32_hi(s[j + 2]),
                                     tf32_hi(s[j + 3]));
        const float4 lo = make_float4(s[j] - h.x, s[j + 1] - h.y, s[j + 2] - h.z, s[j + 3] - h.w);
        const uint32_t o = sw_off(row, j, kFpRows);
        sts4(base + G::PH + o, h);
        sts4(base + G::PL + o, lo);
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    if (it > 0) {  // O rows *= corr (the previous tile's P.V is complete)
      const float c = corr[row];
      if (!__all_sync(0xffffffffu, c == 1.0f)) {
#pragma unroll
        for (int cc = 0; cc < HD / 2; cc += 32) {
          float o[32];
          const uint32_t a = tlane + (uint32_t)(G::OC + half * (HD / 2) + cc);
          tm_ld32(a, o);
          tm_wait_ld(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= c;
          tm_st32(a, o);
        }
        tm_wait_st();
      }
      fence_before();
      __syncthreads();
    }
    if (tid == 0) {  // O += Ph Vh + Ph Vl + Pl Vh
      fence_after();
      constexpr uint32_t idO = fp_idesc(HD);
#pragma unroll
      for (int j = 0; j < kFpKeys / 8; ++j) {
        const uint32_t ao = (uint32_t)((j >> 2) * kFpRows * 128 + (j & 3) * 32);
        const uint32_t bo = (uint32_t)((j >> 2) * HD * 128 + (j & 3) * 32);
        const uint64_t ah = sw128(base + G::PH + ao), al = sw128(base + G::PL + ao);
        const uint64_t bh = sw128(base + G::VH + bo), bl = sw128(base + G::VL + bo);
        mma_ss(tmem + G::OC, ah, bh, idO, (it > 0 || j > 0) ? 1u : 0u);
        mma_ss(tmem + G::OC, ah, bl, idO, 1u);
        mma_ss(tmem + G::OC, al, bh, idO, 1u);
      }
      mma_commit(bar_o);
    }
    ok = __syncthreads_and(fp_wait(bar_o, (uint32_t)(it & 1), abort, p.status)) != 0;
    fence_after();
  }

  // epilogue: O / l (one split) or the split's partial (O, m, l)
  if (warp < 4) {
    rowm[row] = m;
    rowl[row] = l;
  }
  __syncthreads();
  {
    const float lr = rowl[row], mr = rowm[row];
#pragma unroll
    for (int cc = 0; cc < HD / 2; cc += 32) {
      float o[32];
      tm_ld32(tlane + (uint32_t)(G::OC + half * (HD / 2) + cc), o);
      tm_wait_ld(o);
      if (ntile == 0 || !ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.0f;
      }
      if (valid) {
        const int d0 = half * (HD / 2) + cc;
        if (p.NS == 1) {
          float* dst = p.out + ((size_t)tq * p.nh + (size_t)kh * Gq + gq) * HD + d0;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + j) =
                make_float4(o[j] / lr, o[j + 1] / lr, o[j + 2] / lr, o[j + 3] / lr);
        } else {
          float* dst = p.ws + ((((size_t)split * p.nkv + kh) * p.MT + mt) * kFpRows + row) * (HD + 2);
#pragma unroll
          for (int j = 0; j < 32; ++j) dst[d0 + j] = o[j];
          if (half == 0 && cc == 0) {
            dst[HD] = ntile > 0 ? mr : -INFINITY;
            dst[HD + 1] = ntile > 0 ? lr : 0.0f;
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(G::TMEM_COLS)
                 : "memory");
  }
}

// Merge of the splits' partials of one (token, head): weights exp(m_s - M).
__global__ void __launch_bounds__(128) fp_combine_kernel(const float* __restrict__ ws,
                                                         float* __restrict__ out, int nh, int nkv,
                                                         int G, int MT, int NS, int hd) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x / nh, h = blockIdx.x - t * nh, kh = h / G, g = h - kh * G;
  const int rg = t * G + g, mt = rg / kFpRows, row = rg - mt * kFpRows;
  const size_t sstride = (size_t)nkv * MT * kFpRows * (hd + 2);
  const float* e0 = ws + (((size_t)kh * MT + mt) * kFpRows + row) * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < NS; ++s) M = fmaxf(M, e0[s * sstride + hd]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f, ls = 0.0f;
    for (int s = 0; s < NS; ++s) {
      const float* e = e0 + s * sstride;
      const float ms = e[hd];
      const float w = ms == -INFINITY ? 0.0f : expf(ms - M);
      acc = fmaf(w, e[d], acc);
      ls = fmaf(w, e[hd + 1], ls);
    }
    out[((size_t)t * nh + h) * hd + d] = acc / ls;
  }
}

struct FpPlan {
  int G, MT, NS, nkt;
};

FpPlan fp_plan(int T, int nh, int nkv, int p0) {
  FpPlan pl{};
  pl.G = nh / nkv;
  pl.MT = (T * pl.G + kFpRows - 1) / kFpRows;
  pl.nkt = (p0 + T + kFpKeys - 1) / kFpKeys;
  const int per = nkv * pl.MT;
  pl.NS = std::max(1, std::min(sm_count() / std::max(1, per), pl.nkt));
  return pl;
}

template <int HD>
minq_status fp_launch(const FpParams& p, cudaStream_t s) {
  using G = FpGeom<HD>;
  auto k = fp_attn_kernel<HD>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), G::smem));
  MINQ_CUDA_TRY(launch_k(k, dim3(p.NS, p.MT, p.nkv), dim3(kFpThreads), G::smem, s, p));
  return MINQ_OK;
}

}  // namespace

bool prefill_attention_supported(int nh, int nkv, int hd) {
  return (hd == 64 || hd == 128) && nkv > 0 && nh % nkv == 0;
}

size_t prefill_attention_workspace(int T, int nh, int nkv, int hd) {
  if (T <= 0 || nkv <= 0 || nh % nkv) return 0;
  const int G = nh / nkv, MT = (T * G + kFpRows - 1) / kFpRows;
  const int ns = std::max(1, sm_count() / std::max(1, nkv * MT));
  return ns > 1 ? (size_t)ns * nkv * MT * kFpRows * (hd + 2) * sizeof(float) : 0;
}

minq_status launch_prefill_attention(const float* q, const float* kc, const float* vc,
                                     size_t head_stride, int p0, int T, int nh, int nkv, int hd,
                                     float* out, void* ws, size_t ws_bytes, cudaStream_t s,
                                     int* status_word) {
  if (T <= 0 || p0 < 0) return fail(MINQ_ERR_SHAPE, "prefill attention over no tokens");
  if (nkv <= 0 || nh % nkv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  if (!prefill_attention_supported(nh, nkv, hd))
    return fail(MINQ_ERR_SHAPE, "tensor-core prefill attention takes head_dim 64 or 128, not " +
                                    std::to_string(hd));
  if ((uintptr_t)q % 16 || (uintptr_t)kc % 16 || (uintptr_t)vc % 16 || (uintptr_t)out % 16 ||
      head_stride % 4)
    return fail(MINQ_ERR_ARG, "prefill attention: q, k, v, out must be 16-byte aligned");
  const FpPlan pl = fp_plan(T, nh, nkv, p0);
  FpParams p{};
  p.q = q;
  p.kc = kc;
  p.vc = vc;
  p.head_stride = head_stride;
  p.out = out;
  p.p0 = p0;
  p.T = T;
  p.nh = nh;
  p.nkv = nkv;
  p.G = pl.G;
  p.MT = pl.MT;
  p.NS = pl.NS;
  p.nkt = pl.nkt;
  p.scale = 1.0f / sqrtf((float)hd);
  p.status = status_word ? status_word : device_status_word();
  if (pl.NS > 1) {
    const size_t need = (size_t)pl.NS * nkv * pl.MT * kFpRows * (hd + 2) * sizeof(float);
    if (!ws || ws_bytes < need)
      return fail(MINQ_ERR_ARG, "prefill attention workspace too small (need " +
                                    std::to_string(need) + " bytes)");
    p.ws = static_cast<float*>(ws);
  }
  ScopedKTimer timer(KF_ATTENTION, s, 8.0 * nkv * hd * (double)(p0 + T) + 8.0 * T * nh * hd);
  if (hd == 128) MINQ_TRY(fp_launch<128>(p, s));
  else MINQ_TRY(fp_launch<64>(p, s));
  MINQ_LAUNCH_CHECK("fp_attn_kernel");
  if (pl.NS > 1) {
    MINQ_CUDA_TRY(launch_k(fp_combine_kernel, dim3((unsigned)(T * nh)), dim3(std::min(hd, 128)), 0,
                           s, (const float*)p.ws, out, nh, nkv, pl.G, pl.MT, pl.NS, hd));
    MINQ_LAUNCH_CHECK("fp_combine_kernel");
  }
  return MINQ_OK;
}

}  // namespace minq
