// Batch-1 decode step as ONE persistent cooperative kernel (Model::forward_token,
// model.rs:273-318, for a single token), for models whose projections are all
// Q8_0 or all Q4_0 with a fused q|k|v, head_dim 64 or 128, at most 8 query heads
// per KV head and a tied f32 lm_head.
//
// Why one kernel: a decode token is ~250 dependent steps, each far too small to
// fill B200 on its own (a projection is 6-31 MB, 1-5 us of HBM time), so a
// kernel per step spends most of its time launching, ramping up and draining.
// Here every CTA (one per SM) runs the whole token:
//
//   * a producer warp streams this CTA's share of every layer's weights and of
//     every layer's K/V history into a ring of 16 KB shared-memory slots, in
//     the order the consumers use them, without ever waiting on other CTAs:
//     TMA tensor boxes (rows x 32 blocks) for the projections, 1-D bulk copies
//     of TP positions of K and V for attention. It runs ahead across phase and
//     layer boundaries, so HBM keeps streaming while the consumers wait at a
//     grid barrier;
//   * 16 consumer warps execute the phases of each layer:
//       P1 q|k|v = W_qkv rmsnorm(x) + bias                 (rows split over CTAs)
//       P2 attention: CTA = (kv head, split of the history); q/k RMSNorm +
//          RoPE for the new position, the split's online softmax, the new
//          position's k/v appended to the cache by the last split; the last
//          CTA of a kv head to finish merges the splits
//       P3 x = x + W_o att                                  (rows split)
//       P4 h = silu(W_gate rmsnorm(x)) * (W_up rmsnorm(x))  (row pairs split)
//       P5 x = x + W_down h                                 (rows split)
//     with a grid barrier after each phase (time-bounded; a CTA that times out
//     sets the device status word and an abort flag and every CTA stops);
//   * finally the f32 lm_head with the final RMSNorm and a fused argmax
//     (f32::total_cmp order, ties to the lowest index, sampler.rs:10-17),
//     the token and the position written back for the next step.
//
// Every consumer warp waits for and releases every slot in order (a warp
// that skipped slots could reach a slot two phases early, where a parity wait
// cannot tell the phases apart): in projections each warp owns one 4-block
// group of every chunk and a quarter of the rows; in attention each warp owns
// one position of every K/V tile.
//
// The quantized dot products are those of the streaming matvec: exact code ->
// float conversion (byte permute into 2^23 + code), packed f32x2 FMAs, the
// block scale applied once per block (quantize.rs:252-280). Cross-CTA data
// (x, q|k|v, attention output, h, split partials) is read with ld.global.cg
// so no stale L1 line is used after a barrier.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "decode_mk.h"
#include "kernels.h"
#include "matvec_common.cuh"
#include "pipeline.cuh"

namespace minq {

constexpr int kMkCW = 16;                      // consumer warps
constexpr int kMkConsumers = 32 * kMkCW;       // consumer threads
constexpr int kMkThreads = kMkConsumers + 32;  // + the producer warp
constexpr int kMkSlot = 16384;                 // bytes per ring slot
constexpr int kMkMaxS = 12;                    // max ring slots
constexpr int kMkCK = 32;                      // blocks per projection chunk (8 groups of 4)
// Row slots per lane (rows 4k + 2*half + h of a pass): enough for the most
// rows of each format whose box fits a 16 KB slot (Q4_0: 25 single / 12
// pairs, Q8_0: 14 single / 7 pairs).
template <int DT, bool DUAL>
struct MkAccN {
  static constexpr int value = DUAL ? (DT == MINQ_Q4_0 ? 3 : 2) : (DT == MINQ_Q4_0 ? 7 : 4);
};
__host__ __device__ constexpr int mk_acc(int dt, bool dual) {
  return dual ? (dt == MINQ_Q4_0 ? 3 : 2) : (dt == MINQ_Q4_0 ? 7 : 4);
}
constexpr int kMkMiscOff = 256;                // after the full/empty barriers
constexpr int kMkRedOff = 1024;                // projection pass reduction 2 x [8][32][2]
constexpr int kMkScrOff = 5120;                // x / attention scratch, then the ring

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Packed partial dot of one lane's 8 columns of a block (see qmatvec_tma.cu):
// Q8_0: x of the 8 columns in order; Q4_0: (x_even - x_odd/16, x_odd/16) of
// the 4 column pairs, with b = lo + 16*hi the raw code byte.
template <int DT>
__device__ __forceinline__ float2 mk_dot8(uint32_t c0, uint32_t c1, const float4& xa,
                                          const float4& xb) {
  float2 a, s;
  if (DT == MINQ_Q8_0) {
    const uint32_t w0 = c0 ^ 0x80808080u, w1 = c1 ^ 0x80808080u;
    const float2 k = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    a = __fadd2_rn(bytes_to_float2(w0, 0, 1), k);
    s = __fmul2_rn(a, make_float2(xa.x, xa.y));
    a = __fadd2_rn(bytes_to_float2(w0, 2, 3), k);
    s = __ffma2_rn(a, make_float2(xa.z, xa.w), s);
    a = __fadd2_rn(bytes_to_float2(w1, 0, 1), k);
    s = __ffma2_rn(a, make_float2(xb.x, xb.y), s);
    a = __fadd2_rn(bytes_to_float2(w1, 2, 3), k);
    s = __ffma2_rn(a, make_float2(xb.z, xb.w), s);
  } else {
    const uint32_t lo = c0 & 0x0F0F0F0Fu;
    const float2 kl = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    const float2 kb = make_float2(-8388744.0f, -8388744.0f);  // -(2^23 + 136)
    a = __fadd2_rn(bytes_to_float2(lo, 0, 1), kl);
    s = __fmul2_rn(a, make_float2(xa.x, xa.y));
    a = __fadd2_rn(bytes_to_float2(lo, 2, 3), kl);
    s = __ffma2_rn(a, make_float2(xa.z, xa.w), s);
    a = __fadd2_rn(bytes_to_float2(c0, 0, 1), kb);
    s = __ffma2_rn(a, make_float2(xb.x, xb.y), s);
    a = __fadd2_rn(bytes_to_float2(c0, 2, 3), kb);
    s = __ffma2_rn(a, make_float2(xb.z, xb.w), s);
  }
  return s;
}

struct MkRing {
  uint64_t* full;
  uint64_t* empty;
  unsigned char* base;
  int S;
};

// Balanced contiguous share [begin, begin + cnt) of `units` for this CTA.
__device__ __forceinline__ void mk_share(int units, int* begin, int* cnt) {
  const int q = units / (int)gridDim.x, rem = units % (int)gridDim.x;
  const int b = blockIdx.x;
  *begin = b * q + (b < rem ? b : rem);
  *cnt = q + (b < rem ? 1 : 0);
}

// Splits of each kv head's history for a history of L positions: about two
// K/V tiles per split at least, at most p.nsplit (CTAs / kv heads).
__device__ __forceinline__ int mk_nsplit(const MkParams& p, int L) {
  const int tp = 2048 / p.hd;
  const int ntiles = (L + tp - 1) / tp;
  return max(1, min(p.nsplit, (ntiles + 1) / 2));
}

// Attention work item of this CTA: kv head, history tiles [t0, t1), whether
// it also takes the new position. Returns false when the CTA has none.
__device__ __forceinline__ bool mk_attn_item(const MkParams& p, int L, int* kh, int* t0, int* t1,
                                             bool* last) {
  const int ns = mk_nsplit(p, L);
  const int item = blockIdx.x;
  if (item >= p.nkv * ns) return false;
  *kh = item / ns;
  const int sp = item % ns;
  const int tp = 2048 / p.hd;
  const int ntiles = (L + tp - 1) / tp;
  *t0 = (int)(((long long)ntiles * sp) / ns);
  *t1 = (int)(((long long)ntiles * (sp + 1)) / ns);
  *last = sp == ns - 1;
  return true;
}

// ---------------------------------------------------------------- producer

// Wait until slot it % S may be refilled; false on abort or timeout. Lane 0
// decides and the warp follows it, so the producer warp never diverges.
__device__ bool mk_wait_empty(const MkParams& p, const MkRing& r, int it) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const int s = it % r.S;
    const uint32_t parity = ((uint32_t)(it / r.S) & 1u) ^ 1u;
    if (!mbar_try_wait(&r.empty[s], parity)) {
      const uint64_t t0 = global_timer_ns();
      for (;;) {
        if (mbar_try_wait_sleep(&r.empty[s], parity, 20000u)) break;
        if (*reinterpret_cast<volatile int*>(p.abort_flag)) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.status, kDeviceTimeout);
          atomicExch(p.abort_flag, 1);
          ok = 0;
          break;
        }
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int DT, bool DUAL>
__device__ bool mk_produce_mat(const MkParams& p, const MkMat& m, const CUtensorMap* g,
                               const CUtensorMap* u, const MkRing& r, int& it) {
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  constexpr int PITCH = kMkCK * BB;
  const int lane = threadIdx.x & 31;
  int rb, cnt;
  mk_share(m.rows, &rb, &cnt);
  const int passes = (cnt + m.nr - 1) / m.nr;
  for (int j = 0; j < passes; ++j) {
    const int pr0 = (int)(((long long)cnt * j) / passes);
    const int n = (int)(((long long)cnt * (j + 1)) / passes) - pr0;
    const bool big = n == m.nr;
    const uint32_t box = (uint32_t)((big ? m.nr : m.nr_b) * PITCH);
    for (int c = 0; c < m.nchunks; ++c, ++it) {
      if (!mk_wait_empty(p, r, it)) return false;
      if (lane == 0) {
        const int s = it % r.S;
        unsigned char* dst = r.base + (size_t)s * kMkSlot;
        mbar_arrive_expect_tx(&r.full[s], (DUAL ? 2u : 1u) * box);
        const int x = c * (PITCH / 8), y = rb + pr0;  // 8-byte elements
        tma_load_2d_nohint(dst, big ? g : g + 1, x, y, &r.full[s]);
        if (DUAL) tma_load_2d_nohint(dst + m.up_off, big ? u : u + 1, x, y, &r.full[s]);
      }
      __syncwarp();
    }
  }
  return true;
}

__device__ bool mk_produce_attn(const MkParams& p, int li, int L, const MkRing& r, int& it) {
  int kh, t0, t1;
  bool last;
  if (!mk_attn_item(p, L, &kh, &t0, &t1, &last)) return true;
  const int lane = threadIdx.x & 31;
  const int hd = p.hd, tp = 2048 / hd;
  const size_t head_off = (size_t)li * p.cache_layer_stride + (size_t)kh * p.max_seq * hd;
  for (int t = t0; t < t1; ++t, ++it) {
    if (!mk_wait_empty(p, r, it)) return false;
    if (lane == 0) {
      const int s = it % r.S;
      const int p0 = t * tp, np = min(tp, L - p0);
      const uint32_t bytes = (uint32_t)(np * hd * 4);  // hd*4 % 16 == 0
      unsigned char* dst = r.base + (size_t)s * kMkSlot;
      mbar_arrive_expect_tx(&r.full[s], 2u * bytes);
      bulk_g2s(dst, p.kc + head_off + (size_t)p0 * hd, bytes, &r.full[s]);
      bulk_g2s(dst + tp * hd * 4, p.vc + head_off + (size_t)p0 * hd, bytes, &r.full[s]);
    }
    __syncwarp();
  }
  return true;
}

template <int DT>
__device__ void mk_producer(const MkParams& p, const MkRing& r, int L) {
  int it = 0;
  bool ok = !*reinterpret_cast<volatile int*>(p.abort_flag);
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const CUtensorMap* mp = p.maps + (size_t)li * 10;
    ok = mk_produce_mat<DT, false>(p, p.qkv, mp + 0, nullptr, r, it) &&
         mk_produce_attn(p, li, L, r, it) &&
         mk_produce_mat<DT, false>(p, p.o, mp + 2, nullptr, r, it) &&
         mk_produce_mat<DT, true>(p, p.gu, mp + 4, mp + 6, r, it) &&
         mk_produce_mat<DT, false>(p, p.down, mp + 8, nullptr, r, it);
  }
  // Every issued copy lands before the CTA may exit.
  for (int t = max(0, it - r.S); t < it; ++t)
    mbar_wait_timed(&r.full[t % r.S], (uint32_t)(t / r.S) & 1u, p.status);
}

// ---------------------------------------------------------------- consumers

__device__ __forceinline__ void mk_sync() { named_barrier_sync(1, kMkConsumers); }

// Consumer wait for slot it % S. Never leaves the caller's barrier sequence:
// after an abort (or its own timeout, which raises the abort) it returns at
// once and the caller goes on with stale data; every CTA then stops at the
// next grid barrier.
__device__ __forceinline__ void mk_wait_full(const MkParams& p, const MkRing& r, int it) {
  const int s = it % r.S;
  const uint32_t parity = (uint32_t)(it / r.S) & 1u;
  if (mbar_try_wait(&r.full[s], parity)) return;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(&r.full[s], parity, 20000u)) return;
    if (*reinterpret_cast<volatile int*>(p.abort_flag)) return;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(p.status, kDeviceTimeout);
      atomicExch(p.abort_flag, 1);
      return;
    }
  }
}

// Grid barrier over the consumers of all CTAs (monotonic 64-bit counter).
__device__ bool mk_grid_sync(const MkParams& p, unsigned long long target, int* flag) {
  mk_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.bar_ctr, 1ull);
    int ok = 1;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p.bar_ctr) : "memory");
      if (v >= target) break;
      if (*reinterpret_cast<volatile int*>(p.abort_flag)) {
        ok = 0;
        break;
      }
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        atomicOr(p.status, kDeviceTimeout);
        atomicExch(p.abort_flag, 1);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *reinterpret_cast<volatile int*>(flag) = ok;
  }
  mk_sync();
  return *reinterpret_cast<volatile int*>(flag) != 0;
}

// Stage the phase input in shared memory: xs = src (n floats, n % 8 == 0),
// times rmsnorm(src) * gain when gain is set (tensor.rs:219-227), in the
// Q4_0 pair layout when q4. Each thread transforms the groups of 8 it loaded
// itself, so only the sum of squares needs a block-wide step.
__device__ void mk_stage_x(const MkParams& p, float* xs, const float* src, int n,
                           const float* gain, bool q4, float* misc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = n >> 3;
  float4* xs4 = reinterpret_cast<float4*>(xs);
  float inv = 1.0f;
  if (gain) {
    float ss = 0.0f;
    for (int gi = tid; gi < ng; gi += kMkConsumers) {
      const float4 a = ldcg4(src + 8 * gi), b = ldcg4(src + 8 * gi + 4);
      xs4[2 * gi] = a;
      xs4[2 * gi + 1] = b;
      ss = fmaf(a.x, a.x, ss);
      ss = fmaf(a.y, a.y, ss);
      ss = fmaf(a.z, a.z, ss);
      ss = fmaf(a.w, a.w, ss);
      ss = fmaf(b.x, b.x, ss);
      ss = fmaf(b.y, b.y, ss);
      ss = fmaf(b.z, b.z, ss);
      ss = fmaf(b.w, b.w, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) misc[warp] = ss;
    mk_sync();
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kMkCW; ++w) v += misc[w];
    inv = 1.0f / sqrtf(v / (float)n + p.eps);
  }
  const float4* g4 = reinterpret_cast<const float4*>(gain);
  for (int gi = tid; gi < ng; gi += kMkConsumers) {
    float4 a, b;
    if (gain) {
      a = xs4[2 * gi];
      b = xs4[2 * gi + 1];
      const float4 ga = g4[2 * gi], gb = g4[2 * gi + 1];
      a.x = a.x * inv * ga.x; a.y = a.y * inv * ga.y; a.z = a.z * inv * ga.z; a.w = a.w * inv * ga.w;
      b.x = b.x * inv * gb.x; b.y = b.y * inv * gb.y; b.z = b.z * inv * gb.z; b.w = b.w * inv * gb.w;
    } else {
      a = ldcg4(src + 8 * gi);
      b = ldcg4(src + 8 * gi + 4);
    }
    if (q4) {
      const float o0 = a.y * 0.0625f, o1 = a.w * 0.0625f, o2 = b.y * 0.0625f,
                  o3 = b.w * 0.0625f;
      xs4[2 * gi] = make_float4(a.x - o0, a.z - o1, b.x - o2, b.z - o3);
      xs4[2 * gi + 1] = make_float4(o0, o1, o2, o3);
    } else {
      xs4[2 * gi] = a;
      xs4[2 * gi + 1] = b;
    }
  }
  mk_sync();
}

// One projection phase. epi(row, v0, v1) gets the finished row (v1 = up for
// the dual gate/up form).
template <int DT, bool DUAL, class Epi>
__device__ void mk_consume_mat(const MkParams& p, const MkMat& m, const float* xs,
                               const MkRing& r, float* red, int& it, Epi epi) {
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  constexpr int PITCH = kMkCK * BB;
  constexpr int kMkAcc = MkAccN<DT, DUAL>::value;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = warp & 7, rs = warp >> 3;
  const int h = lane >> 4, bi = (lane >> 2) & 3, sub = lane & 3;
  const int nb = m.cols / kBlock;
  int rb, cnt;
  mk_share(m.rows, &rb, &cnt);
  const int passes = (cnt + m.nr - 1) / m.nr;
  for (int j = 0; j < passes; ++j) {
    const int pr0 = (int)(((long long)cnt * j) / passes);
    const int n = (int)(((long long)cnt * (j + 1)) / passes) - pr0;
    float acc[kMkAcc], acc1[DUAL ? kMkAcc : 1];
#pragma unroll
    for (int k = 0; k < kMkAcc; ++k) {
      acc[k] = 0.0f;
      if (DUAL) acc1[k] = 0.0f;
    }
    for (int c = 0; c < m.nchunks; ++c, ++it) {
      const int s = it % r.S;
      mk_wait_full(p, r, it);
      if (c * kMkCK + 4 * grp < nb) {  // nb % 4 == 0: the group is whole or absent
        const int bl = 4 * grp + bi;
        const int bg = c * kMkCK + bl;
        const float4 xa = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub);
        const float4 xb = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub + 4);
        const unsigned char* bp =
            r.base + (size_t)s * kMkSlot + (size_t)(2 * rs + h) * PITCH + bl * BB;
#pragma unroll
        for (int k = 0; k < kMkAcc; ++k) {
          if (4 * k + 2 * rs + h < n) {
            const unsigned char* blk = bp + (size_t)(4 * k) * PITCH;
            const uint32_t* wp =
                reinterpret_cast<const uint32_t*>(blk + 4 + (DT == MINQ_Q8_0 ? 8 : 4) * sub);
            const float d = *reinterpret_cast<const float*>(blk);
            const float2 part = mk_dot8<DT>(wp[0], DT == MINQ_Q8_0 ? wp[1] : 0u, xa, xb);
            acc[k] = fmaf(d, part.x + part.y, acc[k]);
            if (DUAL) {
              const unsigned char* blk1 = blk + m.up_off;
              const uint32_t* wp1 = reinterpret_cast<const uint32_t*>(
                  blk1 + 4 + (DT == MINQ_Q8_0 ? 8 : 4) * sub);
              const float d1 = *reinterpret_cast<const float*>(blk1);
              const float2 part1 = mk_dot8<DT>(wp1[0], DT == MINQ_Q8_0 ? wp1[1] : 0u, xa, xb);
              acc1[k] = fmaf(d1, part1.x + part1.y, acc1[k]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&r.empty[s]);
    }
    // sum over the 16 lanes of each half (4 blocks x 4 column slices), then
    // over the 8 groups in a fixed order; passes alternate between two
    // buffers so one barrier per pass suffices
    float* rb_ = red + (j & 1) * 512;
#pragma unroll
    for (int k = 0; k < kMkAcc; ++k) {
      float v = acc[k], v1 = DUAL ? acc1[k] : 0.0f;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
        if (DUAL) v1 += __shfl_xor_sync(0xffffffffu, v1, o);
      }
      const int row = 4 * k + 2 * rs + h;
      if ((lane & 15) == 0) {
        rb_[(grp * 32 + row) * 2] = v;
        if (DUAL) rb_[(grp * 32 + row) * 2 + 1] = v1;
      }
    }
    mk_sync();
    if (tid < n) {
      float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        v0 += rb_[(g * 32 + tid) * 2];
        if (DUAL) v1 += rb_[(g * 32 + tid) * 2 + 1];
      }
      epi(rb + pr0 + tid, v0, v1);
    }
  }
}

// RMSNorm (optional) + NeoX RoPE of one head held by a warp (model.rs:140-216):
// lane owns pairs (i, i + hd/2), i = lane + 32k. Writes the head to dst.
__device__ void mk_head_prep(const MkParams& p, const float* src, const float* gain, bool rope,
                             int pos, float* dst) {
  const int lane = threadIdx.x & 31, hd = p.hd, half = hd / 2;
  float a[2], b[2];  // hd <= 128: at most 2 pairs per lane
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = lane + 32 * k;
    a[k] = i < half ? ldcg(src + i) : 0.0f;
    b[k] = i < half ? ldcg(src + i + half) : 0.0f;
  }
  if (gain) {
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 2; ++k) ss = fmaf(a[k], a[k], fmaf(b[k], b[k], ss));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + p.eps);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = lane + 32 * k;
      if (i < half) {
        a[k] = a[k] * inv * gain[i];
        b[k] = b[k] * inv * gain[i + half];
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = lane + 32 * k;
    if (i >= half) continue;
    float x1 = a[k], x2 = b[k];
    if (rope) {
      const float c = p.rope_cos[(size_t)pos * half + i];
      const float s = p.rope_sin[(size_t)pos * half + i];
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      x1 = y1;
      x2 = y2;
    }
    dst[i] = x1;
    dst[i + half] = x2;
  }
}

// Online-softmax update of one warp's state with one position (attend,
// model.rs:223-248: s = q.k / sqrt(hd), softmax over positions, sum p v).
// Lane holds dims [DPL*lane, DPL*lane + DPL) of q, k, v and o.
template <int DPL, int GM>
__device__ __forceinline__ void mk_attn_update(const float (&q)[GM][DPL], const float* k,
                                               const float* v, int G, float scale,
                                               float (&m)[GM], float (&l)[GM],
                                               float (&o)[GM][DPL]) {
  const int lane = threadIdx.x & 31;
  float kv[DPL], vv[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    kv[e] = k[DPL * lane + e];
    vv[e] = v[DPL * lane + e];
  }
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      float sv = 0.0f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) sv = fmaf(q[g][e], kv[e], sv);
      sv = warp_sum(sv) * scale;
      const float mn = fmaxf(m[g], sv);
      const float corr = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
      const float pr = expf(sv - mn);
      l[g] = fmaf(l[g], corr, pr);
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pr, vv[e], o[g][e] * corr);
      m[g] = mn;
    }
  }
}

template <int DPL, int GM>
__device__ void mk_consume_attn(const MkParams& p, int li, int L, float* scr, const MkRing& r,
                                int* misc_i, int& it) {
  int kh, t0, t1;
  bool last;
  if (!mk_attn_item(p, L, &kh, &t0, &t1, &last)) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.G, hd = p.hd, tp = 2048 / hd;
  float* qs = scr;                // [G][hd]
  float* knew = qs + G * hd;      // [hd]
  float* vnew = knew + hd;        // [hd]
  float* mg = vnew + hd;          // [16][G]
  float* lg = mg + kMkCW * G;     // [16][G]
  float* og = lg + kMkCW * G;     // [16][G][hd]
  const MkLayerPtrs& lp = p.layers[li];
  const size_t head_off = (size_t)li * p.cache_layer_stride + (size_t)kh * p.max_seq * hd;
  // q heads (q_norm, RoPE at position L); the last split also builds the new
  // k (k_norm, RoPE) and v and appends them to the cache
  if (warp < G) {
    mk_head_prep(p, p.qkv_out + (size_t)(kh * G + warp) * hd, lp.q_norm, true, L,
                 qs + warp * hd);
  } else if (last && warp == G) {
    mk_head_prep(p, p.qkv_out + p.qd + (size_t)kh * hd, lp.k_norm, true, L, knew);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) p.kc[head_off + (size_t)L * hd + i] = knew[i];
  } else if (last && warp == G + 1) {
    for (int i = lane; i < hd; i += 32) {
      const float v = ldcg(p.qkv_out + p.qd + p.kvd + (size_t)kh * hd + i);
      vnew[i] = v;
      p.vc[head_off + (size_t)L * hd + i] = v;
    }
  }
  mk_sync();
  float q[GM][DPL], m[GM], l[GM], o[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      q[g][e] = g < G ? qs[g * hd + DPL * lane + e] : 0.0f;
      o[g][e] = 0.0f;
    }
  }
  for (int t = t0; t < t1; ++t, ++it) {
    const int s = it % r.S;
    mk_wait_full(p, r, it);
    const float* kt = reinterpret_cast<const float*>(r.base + (size_t)s * kMkSlot);
    const float* vt = kt + tp * hd;
    const int np = min(tp, L - t * tp);
    for (int pi = warp; pi < np; pi += kMkCW)
      mk_attn_update<DPL, GM>(q, kt + pi * hd, vt + pi * hd, G, p.scale, m, l, o);
    __syncwarp();
    if (lane == 0) mbar_arrive(&r.empty[s]);
  }
  if (last && warp == 0) mk_attn_update<DPL, GM>(q, knew, vnew, G, p.scale, m, l, o);
  // merge the 16 warps' states
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      if (lane == 0) {
        mg[warp * G + g] = m[g];
        lg[warp * G + g] = l[g];
      }
#pragma unroll
      for (int e = 0; e < DPL; ++e) og[(warp * G + g) * hd + DPL * lane + e] = o[g][e];
    }
  }
  mk_sync();
  const int item = blockIdx.x;
  float* part = p.part + (size_t)item * G * (hd + 2);  // [G][hd + 2]: o, m, l
  for (int idx = tid; idx < G * hd; idx += kMkConsumers) {
    const int g = idx / hd, d = idx % hd;
    float M = -INFINITY;
    for (int w = 0; w < kMkCW; ++w) M = fmaxf(M, mg[w * G + g]);
    float Ls = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < kMkCW; ++w) {
        const float mw = mg[w * G + g];
        if (mw == -INFINITY) continue;
        const float f = expf(mw - M);
        Ls = fmaf(lg[w * G + g], f, Ls);
        O = fmaf(og[(w * G + g) * hd + d], f, O);
      }
    }
    part[g * (hd + 2) + d] = O;
    if (d == 0) {
      part[g * (hd + 2) + hd] = M;
      part[g * (hd + 2) + hd + 1] = Ls;
    }
  }
  // the last split of this kv head to finish merges all of them
  const int ns = mk_nsplit(p, L);
  __threadfence();
  mk_sync();
  if (tid == 0) {
    const int old = atomicAdd(p.head_ctr + kh, 1);
    misc_i[0] = old == ns - 1;
  }
  mk_sync();
  if (misc_i[0]) {
    __threadfence();
    const float* hp = p.part + (size_t)kh * ns * G * (hd + 2);  // items of head kh
    float* mm = scr;             // [ns][G] split maxima, then weights
    float* ll = mm + ns * G;     // [ns][G]
    for (int i = tid; i < ns * G; i += kMkConsumers) {
      const float* e = hp + (size_t)i * (hd + 2);  // i = sp * G + g
      mm[i] = ldcg(e + hd);
      ll[i] = ldcg(e + hd + 1);
    }
    mk_sync();
    if (tid < G) {
      float M = -INFINITY;
      for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, mm[sp * G + tid]);
      float Ls = 0.0f;
      for (int sp = 0; sp < ns; ++sp) {
        const float ms = mm[sp * G + tid];
        const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
        Ls = fmaf(ll[sp * G + tid], f, Ls);
        mm[sp * G + tid] = f;  // weight of the split before the division
      }
      ll[tid] = 1.0f / Ls;    // ll[0..G) reused: 1 / sum (ll no longer read)
    }
    mk_sync();
    for (int idx = tid; idx < G * hd; idx += kMkConsumers) {
      const int g = idx / hd, d = idx % hd;
      float O = 0.0f;
      for (int sp0 = 0; sp0 < ns; sp0 += 8) {  // 8 independent loads in flight
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int sp = sp0 + u;
          v[u] = sp < ns ? ldcg(hp + ((size_t)sp * G + g) * (hd + 2) + d) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (sp0 + u < ns) O = fmaf(v[u], mm[(sp0 + u) * G + g], O);
      }
      p.att[(size_t)(kh * G + g) * hd + d] = O * ll[g];
    }
    if (tid == 0) p.head_ctr[kh] = 0;
  }
}

// f32 lm_head rows of this CTA (tied embedding, model.rs:561-565) with the
// fused argmax; the per-CTA best goes to argmax_part[blockIdx.x].
__device__ void mk_lm_head(const MkParams& p, const float* xs, unsigned long long* best_s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int v0, cnt;
  mk_share(p.vocab, &v0, &cnt);
  const int nvec = p.H >> 2;
  const float4* xs4 = reinterpret_cast<const float4*>(xs);
  unsigned long long best = 0;
  for (int i = warp; i < cnt; i += 2 * kMkCW) {
    const int r0 = v0 + i, r1 = v0 + min(i + kMkCW, cnt - 1);
    const bool two = i + kMkCW < cnt;
    const float4* w0 = reinterpret_cast<const float4*>(p.lm_head + (size_t)r0 * p.H);
    const float4* w1 = reinterpret_cast<const float4*>(p.lm_head + (size_t)r1 * p.H);
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      const float4 xv = xs4[v];
      const float4 wa = __ldcs(w0 + v);
      const float4 wb = __ldcs(w1 + v);
      a0 = fmaf(wa.x, xv.x, a0);
      a0 = fmaf(wa.y, xv.y, a0);
      a0 = fmaf(wa.z, xv.z, a0);
      a0 = fmaf(wa.w, xv.w, a0);
      a1 = fmaf(wb.x, xv.x, a1);
      a1 = fmaf(wb.y, xv.y, a1);
      a1 = fmaf(wb.z, xv.z, a1);
      a1 = fmaf(wb.w, xv.w, a1);
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if (lane == 0) p.logits[r0] = a0;
    unsigned long long pk = argmax_pack(a0, (uint32_t)r0);
    best = pk > best ? pk : best;
    if (two) {
      if (lane == 0) p.logits[r1] = a1;
      pk = argmax_pack(a1, (uint32_t)r1);
      best = pk > best ? pk : best;
    }
  }
  if (lane == 0) best_s[warp] = best;
  mk_sync();
  if (tid == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kMkCW; ++w) b = best_s[w] > b ? best_s[w] : b;
    p.argmax_part[blockIdx.x] = b;
  }
}

template <int DT>
__device__ void mk_consumers(const MkParams& p, unsigned char* sm, const MkRing& r, int L,
                             uint32_t tok, unsigned long long bbase) {
  float* misc = reinterpret_cast<float*>(sm + kMkMiscOff);         // [0..32]: reductions
  int* misc_i = reinterpret_cast<int*>(sm + kMkMiscOff + 160);     // flags
  unsigned long long* best_s = reinterpret_cast<unsigned long long*>(sm + kMkMiscOff + 256);
  float* red = reinterpret_cast<float*>(sm + kMkRedOff);
  float* xs = reinterpret_cast<float*>(sm + kMkScrOff);
  const int G = gridDim.x;
  int it = 0, nbar = 0;
  bool ok = !*reinterpret_cast<volatile int*>(p.abort_flag);
  auto barrier = [&]() { return mk_grid_sync(p, bbase + (unsigned long long)(++nbar) * G, misc_i + 1); };
  const float* xsrc = p.embed + (size_t)tok * p.H;  // residual source before layer 0's o_proj
  constexpr bool Q4 = DT == MINQ_Q4_0;
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const MkLayerPtrs& lp = p.layers[li];
    // P1: q|k|v
    mk_stage_x(p, xs, xsrc, p.H, lp.attn_norm, Q4, misc);
    const float* bias = lp.bias_qkv;
    mk_consume_mat<DT, false>(p, p.qkv, xs, r, red, it, [&](int row, float v, float) {
      p.qkv_out[row] = bias ? v + bias[row] : v;
    });
    if (!(ok = barrier())) break;
    // P2: attention
    if (p.hd == 128) {
      if (p.G <= 4) mk_consume_attn<4, 4>(p, li, L, xs, r, misc_i, it);
      else mk_consume_attn<4, 8>(p, li, L, xs, r, misc_i, it);
    } else {
      if (p.G <= 4) mk_consume_attn<2, 4>(p, li, L, xs, r, misc_i, it);
      else mk_consume_attn<2, 8>(p, li, L, xs, r, misc_i, it);
    }
    if (!(ok = barrier())) break;
    // P3: x = x + W_o att
    mk_stage_x(p, xs, p.att, p.qd, nullptr, Q4, misc);
    const float* res = xsrc;
    mk_consume_mat<DT, false>(p, p.o, xs, r, red, it, [&](int row, float v, float) {
      p.x[row] = ldcg(res + row) + v;
    });
    xsrc = p.x;
    if (!(ok = barrier())) break;
    // P4: h = silu(gate) * up
    mk_stage_x(p, xs, p.x, p.H, lp.ffn_norm, Q4, misc);
    mk_consume_mat<DT, true>(p, p.gu, xs, r, red, it, [&](int row, float g, float u) {
      p.h[row] = silu(g) * u;
    });
    if (!(ok = barrier())) break;
    // P5: x = x + W_down h
    mk_stage_x(p, xs, p.h, p.I, nullptr, Q4, misc);
    mk_consume_mat<DT, false>(p, p.down, xs, r, red, it, [&](int row, float v, float) {
      p.x[row] = ldcg(p.x + row) + v;
    });
    if (!(ok = barrier())) break;
  }
  if (ok && p.want_logits) {
    mk_stage_x(p, xs, p.x, p.H, p.final_norm, false, misc);
    mk_lm_head(p, xs, best_s);
    ok = barrier();
    if (ok && blockIdx.x == 0) {
      unsigned long long b = 0;
      for (int i = threadIdx.x; i < G; i += kMkConsumers) {
        const unsigned long long v = __ldcg(p.argmax_part + i);
        b = v > b ? v : b;
      }
      b = warp_max_u64(b);
      if ((threadIdx.x & 31) == 0) best_s[threadIdx.x >> 5] = b;
      mk_sync();
      if (threadIdx.x == 0) {
        for (int w = 0; w < kMkCW; ++w) b = best_s[w] > b ? best_s[w] : b;
        *p.d_tok = argmax_unpack_index(b);
      }
    }
  }
  if (ok && blockIdx.x == 0 && threadIdx.x == 0) {
    *p.d_pos = L + 1;
    *p.bar_base = bbase + (unsigned long long)nbar * G;
  }
}

template <int DT>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkParams p) {
  extern __shared__ __align__(128) unsigned char sm[];
  MkRing r;
  r.full = reinterpret_cast<uint64_t*>(sm);
  r.empty = r.full + kMkMaxS;
  r.S = p.S;
  r.base = sm + kMkScrOff + (size_t)p.scratch_bytes;
  const int L = *reinterpret_cast<volatile const int*>(p.d_pos);
  const uint32_t tok = *reinterpret_cast<volatile const uint32_t*>(p.d_tok);
  const unsigned long long bbase = *reinterpret_cast<volatile const unsigned long long*>(p.bar_base);
  if (threadIdx.x == 0) {
    for (int s = 0; s < r.S; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], kMkCW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if ((int)threadIdx.x >= kMkConsumers) {
    mk_producer<DT>(p, r, L);
    return;
  }
  mk_consumers<DT>(p, sm, r, L, tok, bbase);
}

// ---------------------------------------------------------------- host

static PFN_cuTensorMapEncodeTiled_v12000 mk_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of a quantized [rows x cols] weight for boxes of box_rows rows x
// 32 blocks, in 8-byte elements (80 of them per Q4_0 chunk, 144 per Q8_0).
static minq_status mk_encode(const void* w, uint64_t rows, uint64_t cols, int dtype,
                             int box_rows, CUtensorMap* out) {
  auto fn = mk_encode_fn();
  if (!fn) return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const uint64_t row_bytes = cols / kBlock * block_bytes(dtype);
  cuuint64_t dims[2] = {row_bytes / 8, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(kMkCK * block_bytes(dtype) / 8), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MINQ_OK;
}

MkMat mk_plan_mat(int dtype, bool dual, uint64_t rows, uint64_t cols, int grid) {
  MkMat m{};
  const int pitch = kMkCK * block_bytes(dtype);
  int nr_max = 0;
  for (int nr = 1; nr <= 4 * mk_acc(dtype, dual); ++nr) {
    const size_t box = ((size_t)nr * pitch + 127) & ~(size_t)127;
    if ((dual ? 2 : 1) * box <= (size_t)kMkSlot) nr_max = nr;
  }
  const uint64_t rmax = (rows + grid - 1) / grid;
  const uint64_t passes = (rmax + nr_max - 1) / nr_max;
  m.rows = (int)rows;
  m.cols = (int)cols;
  m.nr = (int)((rmax + passes - 1) / passes);
  m.nr_b = m.nr > 1 ? m.nr - 1 : 1;
  m.nchunks = (int)((cols / kBlock + kMkCK - 1) / kMkCK);
  m.up_off = dual ? (int)(((size_t)m.nr * pitch + 127) & ~(size_t)127) : 0;
  return m;
}

minq_status mk_encode_pair(const void* w, uint64_t rows, uint64_t cols, int dtype, const MkMat& m,
                           CUtensorMap* out2) {
  MINQ_TRY(mk_encode(w, rows, cols, dtype, m.nr, &out2[0]));
  MINQ_TRY(mk_encode(w, rows, cols, dtype, m.nr_b, &out2[1]));
  return MINQ_OK;
}

size_t mk_scratch_bytes(int H, int I, int qd, int G, int hd) {
  const size_t xs = (size_t)std::max({H, I, qd}) * 4;
  const size_t att = ((size_t)G * hd + 2 * hd + 2 * kMkCW * G + (size_t)kMkCW * G * hd) * 4;
  return (std::max(xs, att) + 127) & ~(size_t)127;
}

int mk_ring_slots(size_t scratch_bytes) {
  const size_t avail = 227 * 1024 - kMkScrOff - scratch_bytes;
  return (int)std::min<size_t>(kMkMaxS, avail / kMkSlot);
}

size_t mk_smem_bytes(size_t scratch_bytes, int S) {
  return kMkScrOff + scratch_bytes + (size_t)S * kMkSlot;
}

template <int DT>
static minq_status mk_launch_inst(const MkParams& p, int grid, size_t smem, cudaStream_t s) {
  auto k = decode_mk_kernel<DT>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
  int per_sm = 0;
  MINQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kMkThreads, smem));
  if (per_sm < 1)
    return fail(MINQ_ERR_CUDA, "decode megakernel does not fit on an SM (" +
                                   std::to_string(smem) + " bytes of shared memory)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MINQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, p));
  MINQ_LAUNCH_CHECK("decode_mk_kernel");
  return MINQ_OK;
}

minq_status launch_decode_mk(const MkParams& p, int dtype, int grid, size_t smem,
                             cudaStream_t s) {
  if (dtype == MINQ_Q8_0) return mk_launch_inst<MINQ_Q8_0>(p, grid, smem, s);
  return mk_launch_inst<MINQ_Q4_0>(p, grid, smem, s);
}

}  // namespace minq
