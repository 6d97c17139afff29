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
//   * four producer warps stream this CTA's share of every layer's weights and
//     of every layer's K/V history into an 8-slot ring of 16 KB shared-memory
//     tiles with cp.async (16-byte pieces; the slot's full mbarrier tracks them
//     through cp.async.mbarrier.arrive), in the order the consumers use them
//     and without waiting on other CTAs: projection tiles are rows x 32 blocks
//     of the reference's row-major blocks, attention tiles TP positions of K
//     and V. Producer k owns the tiles k, k + 4, ... and so its own slots. The
//     producers run ahead across phase and layer boundaries, so HBM keeps
//     streaming while the consumers wait at a grid barrier. (One CTA per SM
//     issuing TMA copies was measured at half of the HBM bandwidth; cp.async
//     from several warps sustains it.)
//   * 16 consumer warps execute the phases of each layer:
//       P1 q|k|v = W_qkv rmsnorm(x) + bias                 (rows split over CTAs)
//       P2 attention: CTA = (kv head, split of the history); q/k RMSNorm +
//          RoPE for the new position, the split's online softmax, the new
//          position's k/v appended to the cache by the last split; the
//          splits of a head then meet at a per-head counter and each merges
//          a slice of the head's outputs
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
// group of every chunk and a quarter of the rows; in attention the 16 warps
// cooperate on each step of up to 32 positions (scores, softmax, p v).
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

constexpr int kMkCW = 16;                      // warps
constexpr int kMkConsumers = 32 * kMkCW;       // threads (all of them load and compute)
constexpr int kMkProducers = 4;                // copy warps; warp k issues tiles k, k + 4, ...
constexpr int kMkThreads = kMkConsumers + 32 * kMkProducers;
constexpr int kMkSlot = 16384;                 // bytes per ring slot
constexpr int kMkS = 8;                        // ring slots (a multiple of kMkProducers)
static_assert(kMkS % kMkProducers == 0, "each producer warp owns its own slots");
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
constexpr int kMkMiscOff = 256;                // small reductions and flags
constexpr int kMkCtaOff = 768;                 // the CTA's plan (MkCta)
constexpr int kMkRedOff = 1024;                // projection pass reduction 2 x [8][32][2]
constexpr int kMkRopeOff = 5120;               // cos | sin of this position's RoPE row
constexpr int kMkScrOff = 5632;                // x / attention scratch, then the ring

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

// ---------------------------------------------------------------- feed
//
// Every thread of the CTA copies its share of each tile with cp.async
// (16-byte pieces, one commit group per tile), kMkS - 1 tiles ahead of the
// tile being computed on, in the order the phases use them. The tile
// sequence runs across phase and layer boundaries, so the next phase's
// weights are already streaming while the CTA waits at a grid barrier.
// (With one CTA per SM, copies issued by all 512 threads sustain the full
// HBM bandwidth; a single TMA-issuing warp was measured at half of it.)

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Rows of this CTA in a projection and its passes of at most m.nr rows.
struct MkShare {
  int rb, cnt, passes;
};
__device__ __forceinline__ MkShare mk_mat_share(const MkMat& m) {
  MkShare s;
  mk_share(m.rows, &s.rb, &s.cnt);
  s.passes = (s.cnt + m.nr - 1) / m.nr;
  return s;
}
__device__ __forceinline__ int mk_pass_row(const MkShare& s, int j) {
  return (int)(((long long)s.cnt * j) / s.passes);
}

// This CTA's plan for the launch (the same for every layer), computed once
// into shared memory: row shares of the four projections and the attention
// work item. Phases: 0 q|k|v, 1 attention, 2 o, 3 gate/up, 4 down.
struct MkCta {
  MkShare sh[5];   // projections (index 1 unused)
  int tiles[5];    // tiles of each phase
  int kh, t0, t1, last;
};

__device__ __forceinline__ const MkMat& mk_mat(const MkParams& p, int ph) {
  return ph == 0 ? p.qkv : ph == 2 ? p.o : ph == 3 ? p.gu : p.down;
}

__device__ void mk_cta_plan(const MkParams& p, int L, MkCta* c) {
  for (int ph = 0; ph < 5; ++ph) {
    if (ph == 1) continue;
    const MkMat& m = mk_mat(p, ph);
    c->sh[ph] = mk_mat_share(m);
    c->tiles[ph] = c->sh[ph].passes * m.nchunks;
  }
  int kh = 0, t0 = 0, t1 = 0;
  bool last = false;
  const bool has = mk_attn_item(p, L, &kh, &t0, &t1, &last);
  c->kh = kh;
  c->t0 = t0;
  c->t1 = has ? t1 : t0;
  c->last = has && last;
  c->tiles[1] = c->t1 - c->t0;
}

struct MkFeed {
  unsigned char* ring;
  uint64_t* full;   // [kMkS]: the producer lanes' copies of the slot's tile landed
  uint64_t* empty;  // [kMkS]: every consumer warp released the slot
  int li, ph, idx;  // next tile to issue: layer, phase, index in the phase
  int issued;       // tiles issued so far (slot = issued % kMkS)
  int j, c;         // projection pass and chunk of the next tile
  int pr0, n;       // rows of that pass
};

__device__ __forceinline__ void mk_feed_pass(MkFeed& f, const MkShare& sh) {
  f.pr0 = mk_pass_row(sh, f.j);
  f.n = mk_pass_row(sh, f.j + 1) - f.pr0;
}

// Producer wait until slot `it % kMkS` may be refilled; false on abort or
// timeout. Lane 0 decides and the warp follows it.
__device__ bool mk_wait_empty(const MkParams& p, const MkFeed& f, int it) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const int s = it % kMkS;
    const uint32_t parity = ((uint32_t)(it / kMkS) & 1u) ^ 1u;
    if (!mbar_try_wait(&f.empty[s], parity)) {
      const uint64_t t0 = global_timer_ns();
      for (;;) {
        if (mbar_try_wait_sleep(&f.empty[s], parity, 2000u)) break;
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

// Producer: copy the next tile into its slot with the warp's 32 lanes, then
// have the slot's full barrier track the copies (cp.async.mbarrier.arrive).
// Projection tiles: lane l copies 16-byte pieces l, l + 32, ... of each row
// chunk (40 pieces for Q4_0, 72 for Q8_0), the up rows of the gate/up phase
// after the gate rows. Attention tiles: pieces l, l + 32, ... of K and of V.
// Returns false when every tile is issued (or on abort).
// Advance the iterator past phases without tiles; false past the last layer.
__device__ __forceinline__ bool mk_feed_settle(const MkParams& p, MkFeed& f, const MkCta* cta) {
  while (f.li < p.n_layers && f.idx >= cta->tiles[f.ph]) {
    f.idx = 0;
    if (++f.ph == 5) {
      f.ph = 0;
      ++f.li;
    }
    f.j = 0;
    f.c = 0;
    if (f.ph != 1) mk_feed_pass(f, cta->sh[f.ph]);
  }
  return f.li < p.n_layers;
}

// Step the iterator over one tile without copying it.
__device__ __forceinline__ void mk_feed_skip(const MkParams& p, MkFeed& f, const MkCta* cta) {
  if (f.ph != 1 && ++f.c == mk_mat(p, f.ph).nchunks) {
    f.c = 0;
    if (++f.j < cta->sh[f.ph].passes) mk_feed_pass(f, cta->sh[f.ph]);
  }
  ++f.idx;
  ++f.issued;
}

// Producer warp: copy the current tile into its slot with the warp's 32
// lanes, then have the slot's full barrier track the copies
// (cp.async.mbarrier.arrive). Projection tiles: the rows x 16-byte pieces of
// the row chunk (40 pieces for Q4_0, 72 for Q8_0) flattened over the lanes,
// the up rows of the gate/up phase after the gate rows. Attention tiles: the
// pieces of K and of V. False on abort.
template <int DT>
__device__ bool mk_issue(const MkParams& p, MkFeed& f, const MkCta* cta, int L) {
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  constexpr int PITCH = kMkCK * BB;
  constexpr int PPR = PITCH / 16;  // pieces of a full row chunk
  const int lane = threadIdx.x & 31;
  if (!mk_wait_empty(p, f, f.issued)) return false;
  const int slot = f.issued % kMkS;
  unsigned char* dst = f.ring + (size_t)slot * kMkSlot;
  const MkLayerPtrs& lp = p.layers[f.li];
  if (f.ph == 1) {
    const int hd = p.hd, tp = 2048 / hd;
    const int p0 = (cta->t0 + f.idx) * tp, np = min(tp, L - p0);
    const size_t off = (size_t)f.li * p.cache_layer_stride + (size_t)cta->kh * p.max_seq * hd +
                       (size_t)p0 * hd;
    const int pieces = np * hd / 4;  // 16-byte pieces of K (and of V)
    for (int i = lane; i < pieces; i += 32) {
      cp_async16(dst + i * 16, p.kc + off + i * 4);
      cp_async16(dst + tp * hd * 4 + i * 16, p.vc + off + i * 4);
    }
  } else {
    const bool dual = f.ph == 3;
    const MkMat& m = mk_mat(p, f.ph);
    const uint8_t* w0 = f.ph == 0 ? lp.w_qkv : f.ph == 2 ? lp.w_o : dual ? lp.w_gate : lp.w_down;
    const int nb = m.cols / kBlock;
    const int ppr = min(kMkCK, nb - f.c * kMkCK) * BB / 16;  // pieces per row (nb % 4 == 0)
    const size_t row_bytes = (size_t)nb * BB;
    const size_t first = (size_t)(cta->sh[f.ph].rb + f.pr0) * row_bytes + (size_t)f.c * PITCH;
    const int n = f.n, total = (dual ? 2 : 1) * n * ppr;
    for (int i = lane; i < total; i += 32) {
      const int r = ppr == PPR ? i / PPR : i / ppr;  // constant divisor for full chunks
      const int pc = i - r * ppr;
      const bool up = dual && r >= n;
      const int row = up ? r - n : r;
      cp_async16(dst + (up ? m.up_off : 0) + row * PITCH + pc * 16,
                 (up ? lp.w_up : w0) + first + (size_t)row * row_bytes + pc * 16);
    }
  }
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&f.full[slot]))
               : "memory");
  mk_feed_skip(p, f, cta);
  return true;
}

// Producer warp k (of kMkProducers) issues the tiles k, k + kMkProducers, ...
// Because kMkS is a multiple of kMkProducers it alone refills those slots.
template <int DT>
__device__ void mk_producer(const MkParams& p, MkFeed& f, const MkCta* cta, int L) {
  const int k = ((int)threadIdx.x - kMkConsumers) >> 5;
  if (!*reinterpret_cast<volatile int*>(p.abort_flag)) {
    while (mk_feed_settle(p, f, cta)) {
      if (f.issued % kMkProducers == k) {
        if (!mk_issue<DT>(p, f, cta, L)) break;
      } else {
        mk_feed_skip(p, f, cta);
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight at exit
}

// Consumer wait for the tile `it`; never leaves the caller's barrier
// sequence: after an abort (or its own timeout, which raises the abort) it
// returns at once with stale data, and every CTA stops at the next grid
// barrier.
__device__ const unsigned char* mk_next_tile(const MkParams& p, const MkFeed& f, int it) {
  const int s = it % kMkS;
  const uint32_t parity = (uint32_t)(it / kMkS) & 1u;
  if (!mbar_try_wait(&f.full[s], parity)) {
    const uint64_t t0 = global_timer_ns();
    for (;;) {
      if (mbar_try_wait_sleep(&f.full[s], parity, 2000u)) break;
      if (*reinterpret_cast<volatile int*>(p.abort_flag)) break;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        atomicOr(p.status, kDeviceTimeout);
        atomicExch(p.abort_flag, 1);
        break;
      }
    }
  }
  return f.ring + (size_t)s * kMkSlot;
}

// The warp is done with tile `it`.
__device__ __forceinline__ void mk_release(const MkFeed& f, int it) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&f.empty[it % kMkS]);
}

// ---------------------------------------------------------------- consumers

__device__ __forceinline__ void mk_sync() { named_barrier_sync(1, kMkConsumers); }

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
__device__ void mk_consume_mat(const MkParams& p, const MkMat& m, const float* xs, MkFeed& f,
                               const MkCta* cta, int L, float* red, int& it, Epi epi) {
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
      const unsigned char* tile = mk_next_tile(p, f, it);
      if (c * kMkCK + 4 * grp < nb) {  // nb % 4 == 0: the group is whole or absent
        const int bl = 4 * grp + bi;
        const int bg = c * kMkCK + bl;
        const float4 xa = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub);
        const float4 xb = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub + 4);
        const unsigned char* bp = tile + (size_t)(2 * rs + h) * PITCH + bl * BB;
        // all of the lane's code words and scales first (rows past the pass
        // read nothing and count as zero), then the arithmetic: the loads of
        // every row slot are in flight together
        constexpr int NW = DT == MINQ_Q8_0 ? 2 : 1;
        constexpr int NM = DUAL ? 2 : 1;
        uint32_t cw[kMkAcc][NM][NW];
        float dd[kMkAcc][NM];
#pragma unroll
        for (int k = 0; k < kMkAcc; ++k) {
          const bool ok = 4 * k + 2 * rs + h < n;
#pragma unroll
          for (int mm = 0; mm < NM; ++mm) {
            const unsigned char* blk = bp + (size_t)(4 * k) * PITCH + (mm ? m.up_off : 0);
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(blk + 4 + 4 * NW * sub);
            dd[k][mm] = ok ? *reinterpret_cast<const float*>(blk) : 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) cw[k][mm][w] = ok ? wp[w] : 0u;
          }
        }
#pragma unroll
        for (int k = 0; k < kMkAcc; ++k) {
          const float2 part = mk_dot8<DT>(cw[k][0][0], NW == 2 ? cw[k][0][NW - 1] : 0u, xa, xb);
          acc[k] = fmaf(dd[k][0], part.x + part.y, acc[k]);
          if (DUAL) {
            const float2 part1 =
                mk_dot8<DT>(cw[k][NM - 1][0], NW == 2 ? cw[k][NM - 1][NW - 1] : 0u, xa, xb);
            acc1[k] = fmaf(dd[k][NM - 1], part1.x + part1.y, acc1[k]);
          }
        }
      }
      mk_release(f, it);
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
                             const float* rope_cs, float* dst) {
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
      const float c = rope_cs[i];         // cos / sin of this position (shared memory)
      const float s = rope_cs[half + i];
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      x1 = y1;
      x2 = y2;
    }
    dst[i] = x1;
    dst[i + half] = x2;
  }
}

// Shared-memory layout of the attention phase (in the scratch region).
struct MkAttnSmem {
  float* qs;    // [G][hd]   RoPE'd (and normed) query heads
  float* knew;  // [hd]      the new position's key (last split)
  float* vnew;  // [hd]
  float* sc;    // [G][32]   scores of the tile
  float* pp;    // [G][32]   softmax numerators of the tile
  float* corr;  // [G]       rescale of the running output
};

// One step of attend (model.rs:223-248: s = q.k / sqrt(hd), softmax over
// positions, o = sum p v) over up to 32 positions held in shared memory:
// positions j < base1 are rows j of (k0, v0) (j < n0), positions j >= base1
// rows j - base1 of (k1, v1) (j - base1 < n1). As an online softmax: (A)
// warp w scores positions w and w + 16 for every head, (B) warp g < G
// updates head g's running max m and sum l and forms the numerators, (C)
// every thread rescales and accumulates its outputs (head, dim) =
// (idx / hd, idx % hd) for idx = tid, tid + 512. m, l live in warp g's lanes
// (replicated); o in the owning thread.
template <int DPL, int GM>
__device__ void mk_attn_step(const MkParams& p, const MkAttnSmem& a, const float (&q)[GM][DPL],
                             const float* k0, const float* v0, int n0, const float* k1,
                             const float* v1, int n1, int base1, float& m, float& l,
                             float (&o)[2]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.G, hd = p.hd;
  // (A) scores
  float sv[2][GM];
#pragma unroll
  for (int rep = 0; rep < 2; ++rep) {
    const int j = warp + 16 * rep;
    const bool t1 = j >= base1;
    const int r = t1 ? j - base1 : j;
    const bool ok = r < (t1 ? n1 : n0);
    const float* kr = (t1 ? k1 : k0) + (ok ? r : 0) * hd;
    float kv[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) kv[e] = ok ? kr[DPL * lane + e] : 0.0f;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      sv[rep][g] = 0.0f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) sv[rep][g] = fmaf(q[g][e], kv[e], sv[rep][g]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int rep = 0; rep < 2; ++rep)
#pragma unroll
      for (int g = 0; g < GM; ++g) sv[rep][g] += __shfl_xor_sync(0xffffffffu, sv[rep][g], off);
  if (lane < GM && lane < G) {
#pragma unroll
    for (int rep = 0; rep < 2; ++rep) {
      float v = sv[rep][0];
#pragma unroll
      for (int g = 1; g < GM; ++g) v = lane == g ? sv[rep][g] : v;
      a.sc[lane * 32 + warp + 16 * rep] = v * p.scale;
    }
  }
  mk_sync();
  // (B) online softmax per head
  if (warp < G) {
    const bool t1 = lane >= base1;
    const bool ok = (t1 ? lane - base1 : lane) < (t1 ? n1 : n0);
    const float s_ = ok ? a.sc[warp * 32 + lane] : -INFINITY;
    const float mt = warp_max(s_);
    const float mn = fmaxf(m, mt);
    const float c = m == -INFINITY ? 0.0f : expf(m - mn);
    const float pr = s_ == -INFINITY ? 0.0f : expf(s_ - mn);
    l = fmaf(l, c, warp_sum(pr));
    m = mn;
    a.pp[warp * 32 + lane] = pr;
    if (lane == 0) a.corr[warp] = c;
  }
  mk_sync();
  // (C) o = o * corr + sum_j p_j v_j
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int idx = tid + kMkConsumers * u;
    if (idx < G * hd) {
      const int g = idx / hd, d = idx - g * hd;
      const float* pg = a.pp + g * 32;
      const float* va = v0 + d;
      const float* vb = v1 + d;
      float acc = o[u] * a.corr[g], acc2 = 0.0f;
      int j = 0;
#pragma unroll 4
      for (; j + 1 < n0; j += 2) {
        acc = fmaf(pg[j], va[j * hd], acc);
        acc2 = fmaf(pg[j + 1], va[(j + 1) * hd], acc2);
      }
      if (j < n0) acc = fmaf(pg[j], va[j * hd], acc);
      pg += base1;
#pragma unroll 4
      for (j = 0; j + 1 < n1; j += 2) {
        acc = fmaf(pg[j], vb[j * hd], acc);
        acc2 = fmaf(pg[j + 1], vb[(j + 1) * hd], acc2);
      }
      if (j < n1) acc = fmaf(pg[j], vb[j * hd], acc);
      o[u] = acc + acc2;
    }
  }
}

template <int DT, int DPL, int GM>
__device__ void mk_consume_attn(const MkParams& p, int li, int L, float* scr, MkFeed& f,
                                const MkCta* cta, const float* rope_cs, int* misc_i, int& it) {
  int kh, t0, t1;
  bool last;
  if (!mk_attn_item(p, L, &kh, &t0, &t1, &last)) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.G, hd = p.hd, tp = 2048 / hd;
  MkAttnSmem a;
  a.qs = scr;
  a.knew = a.qs + G * hd;
  a.vnew = a.knew + hd;
  a.sc = a.vnew + hd;
  a.pp = a.sc + 32 * G;
  a.corr = a.pp + 32 * G;
  const MkLayerPtrs& lp = p.layers[li];
  const size_t head_off = (size_t)li * p.cache_layer_stride + (size_t)kh * p.max_seq * hd;
  // q heads (q_norm, RoPE at position L); the last split also builds the new
  // k (k_norm, RoPE) and v and appends them to the cache
  if (warp < G) {
    mk_head_prep(p, p.qkv_out + (size_t)(kh * G + warp) * hd, lp.q_norm, true, rope_cs,
                 a.qs + warp * hd);
  } else if (last && warp == G) {
    mk_head_prep(p, p.qkv_out + p.qd + (size_t)kh * hd, lp.k_norm, true, rope_cs, a.knew);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) p.kc[head_off + (size_t)L * hd + i] = a.knew[i];
  } else if (last && warp == G + 1) {
    for (int i = lane; i < hd; i += 32) {
      const float v = ldcg(p.qkv_out + p.qd + p.kvd + (size_t)kh * hd + i);
      a.vnew[i] = v;
      p.vc[head_off + (size_t)L * hd + i] = v;
    }
  }
  mk_sync();
  float q[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < DPL; ++e) q[g][e] = g < G ? a.qs[g * hd + DPL * lane + e] : 0.0f;
  float m = -INFINITY, l = 0.0f, o[2] = {0.0f, 0.0f};
  // two 16-position tiles per step for head_dim 128, one 32-position tile for 64
  const int per_step = 32 / tp;
  for (int t = t0; t < t1; t += per_step) {
    const float* ka = reinterpret_cast<const float*>(mk_next_tile(p, f, it));
    const int na = min(tp, L - t * tp);
    const float* kb = ka;
    int nb_ = 0;
    if (per_step == 2 && t + 1 < t1) {
      kb = reinterpret_cast<const float*>(mk_next_tile(p, f, it + 1));
      nb_ = min(tp, L - (t + 1) * tp);
    }
    mk_attn_step<DPL, GM>(p, a, q, ka, ka + tp * hd, na, kb, kb + tp * hd, nb_, tp, m, l, o);
    mk_release(f, it);
    ++it;
    if (nb_ > 0) {
      mk_release(f, it);
      ++it;
    }
  }
  if (last) mk_attn_step<DPL, GM>(p, a, q, a.knew, a.vnew, 1, a.knew, a.vnew, 0, 32, m, l, o);
  // this split's partial: unnormalised o, running max m and sum l per head
  const int item = blockIdx.x;
  float* part = p.part + (size_t)item * G * (hd + 2);  // [G][hd + 2]: o, m, l
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int idx = tid + kMkConsumers * u;
    if (idx < G * hd) {
      const int g = idx / hd, d = idx - g * hd;
      part[g * (hd + 2) + d] = o[u];
    }
  }
  if (warp < G && lane == 0) {
    part[warp * (hd + 2) + hd] = m;
    part[warp * (hd + 2) + hd + 1] = l;
  }
  // every split of this kv head waits for the others (an arrival counter per
  // head, reset after the next grid barrier), then merges its own slice of
  // the head's G * hd outputs from all splits' partials
  const int ns = mk_nsplit(p, L);
  const int sp = item - kh * ns;
  __threadfence();
  mk_sync();
  if (tid == 0) {
    atomicAdd(p.head_ctr + kh, 1);
    const uint64_t tw = global_timer_ns();
    for (;;) {
      int v;
      asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p.head_ctr + kh) : "memory");
      if (v >= ns) break;
      if (*reinterpret_cast<volatile int*>(p.abort_flag)) break;
      if (global_timer_ns() - tw > kWaitLimitNs) {
        atomicOr(p.status, kDeviceTimeout);
        atomicExch(p.abort_flag, 1);
        break;
      }
    }
    __threadfence();
  }
  mk_sync();
  const int GH = G * hd;
  const int o0 = (int)((long long)GH * sp / ns), o1 = (int)((long long)GH * (sp + 1) / ns);
  const int nout = o1 - o0;
  const int g0 = o0 / hd, ng = (o1 - 1) / hd - g0 + 1;  // heads the slice touches
  const float* hp = p.part + (size_t)kh * ns * G * (hd + 2);
  float* mm = scr;             // [ns][ng] split maxima, then weights
  float* ll = mm + ns * ng;    // [ns][ng]
  float* inv = ll + ns * ng;   // [ng]
  float* vals = inv + ng;      // [ns][nout] weighted partial outputs
  for (int i = tid; i < ns * ng; i += kMkConsumers) {
    const int s_ = i / ng, gg = i - s_ * ng;
    const float* e = hp + ((size_t)s_ * G + g0 + gg) * (hd + 2);
    mm[i] = ldcg(e + hd);
    ll[i] = ldcg(e + hd + 1);
  }
  mk_sync();
  if (tid < ng) {
    float M = -INFINITY;
    for (int s_ = 0; s_ < ns; ++s_) M = fmaxf(M, mm[s_ * ng + tid]);
    float Ls = 0.0f;
    for (int s_ = 0; s_ < ns; ++s_) {
      const float ms = mm[s_ * ng + tid];
      const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
      Ls = fmaf(ll[s_ * ng + tid], f, Ls);
      mm[s_ * ng + tid] = f;
    }
    inv[tid] = 1.0f / Ls;
  }
  mk_sync();
  for (int i = tid; i < ns * nout; i += kMkConsumers) {
    const int s_ = i / nout, oi = i - s_ * nout;
    const int g = (o0 + oi) / hd, d = (o0 + oi) - g * hd;
    vals[i] = ldcg(hp + ((size_t)s_ * G + g) * (hd + 2) + d) * mm[s_ * ng + g - g0];
  }
  mk_sync();
  for (int oi = tid; oi < nout; oi += kMkConsumers) {
    const int g = (o0 + oi) / hd, d = (o0 + oi) - g * hd;
    float O = 0.0f;
    for (int s_ = 0; s_ < ns; ++s_) O += vals[s_ * nout + oi];
    p.att[(size_t)(kh * G + g) * hd + d] = O * inv[g - g0];
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
__device__ void mk_consumers(const MkParams& p, unsigned char* sm, MkFeed& f, const MkCta* cta,
                             int L,
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
  // this position's RoPE row (model.rs:170-186 tables), used by every layer
  float* rope_cs = reinterpret_cast<float*>(sm + kMkRopeOff);
  {
    const int half = p.hd / 2;
    for (int i = threadIdx.x; i < 2 * half; i += kMkConsumers)
      rope_cs[i] = i < half ? p.rope_cos[(size_t)L * half + i] : p.rope_sin[(size_t)L * half + i - half];
  }
  constexpr bool Q4 = DT == MINQ_Q4_0;
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const MkLayerPtrs& lp = p.layers[li];
    // P1: q|k|v
    mk_stage_x(p, xs, xsrc, p.H, lp.attn_norm, Q4, misc);
    const float* bias = lp.bias_qkv;
    mk_consume_mat<DT, false>(p, p.qkv, xs, f, cta, L, red, it, [&](int row, float v, float) {
      p.qkv_out[row] = bias ? v + bias[row] : v;
    });
    if (!(ok = barrier())) break;
    // P2: attention
    if (p.hd == 128) {
      if (p.G <= 4) mk_consume_attn<DT, 4, 4>(p, li, L, xs, f, cta, rope_cs, misc_i, it);
      else mk_consume_attn<DT, 4, 8>(p, li, L, xs, f, cta, rope_cs, misc_i, it);
    } else {
      if (p.G <= 4) mk_consume_attn<DT, 2, 4>(p, li, L, xs, f, cta, rope_cs, misc_i, it);
      else mk_consume_attn<DT, 2, 8>(p, li, L, xs, f, cta, rope_cs, misc_i, it);
    }
    if (!(ok = barrier())) break;
    // P3: x = x + W_o att (every split is past its head's counter now)
    if (blockIdx.x < (unsigned)p.nkv && threadIdx.x == 0) p.head_ctr[blockIdx.x] = 0;
    mk_stage_x(p, xs, p.att, p.qd, nullptr, Q4, misc);
    const float* res = xsrc;
    mk_consume_mat<DT, false>(p, p.o, xs, f, cta, L, red, it, [&](int row, float v, float) {
      p.x[row] = ldcg(res + row) + v;
    });
    xsrc = p.x;
    if (!(ok = barrier())) break;
    // P4: h = silu(gate) * up
    mk_stage_x(p, xs, p.x, p.H, lp.ffn_norm, Q4, misc);
    mk_consume_mat<DT, true>(p, p.gu, xs, f, cta, L, red, it, [&](int row, float g, float u) {
      p.h[row] = silu(g) * u;
    });
    if (!(ok = barrier())) break;
    // P5: x = x + W_down h
    mk_stage_x(p, xs, p.h, p.I, nullptr, Q4, misc);
    mk_consume_mat<DT, false>(p, p.down, xs, f, cta, L, red, it, [&](int row, float v, float) {
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
  const int L = *reinterpret_cast<volatile const int*>(p.d_pos);
  const uint32_t tok = *reinterpret_cast<volatile const uint32_t*>(p.d_tok);
  const unsigned long long bbase = *reinterpret_cast<volatile const unsigned long long*>(p.bar_base);
  MkCta* cta = reinterpret_cast<MkCta*>(sm + kMkCtaOff);
  if (threadIdx.x == 0) mk_cta_plan(p, L, cta);
  __syncthreads();
  MkFeed f;
  f.ring = sm + kMkScrOff + (size_t)p.scratch_bytes;
  f.full = reinterpret_cast<uint64_t*>(sm);
  f.empty = f.full + kMkS;
  f.li = 0;
  f.ph = 0;
  f.idx = 0;
  f.issued = 0;
  f.j = 0;
  f.c = 0;
  mk_feed_pass(f, cta->sh[0]);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkS; ++s) {
      mbar_init(&f.full[s], 32);     // the issuing producer warp's lanes (cp.async.mbarrier.arrive)
      mbar_init(&f.empty[s], kMkCW);  // every consumer warp
    }
    mbar_fence_init();
  }
  __syncthreads();
  if ((int)threadIdx.x >= kMkConsumers) {
    mk_producer<DT>(p, f, cta, L);
    return;
  }
  mk_consumers<DT>(p, sm, f, cta, L, tok, bbase);
}

// ---------------------------------------------------------------- host

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
  m.nchunks = (int)((cols / kBlock + kMkCK - 1) / kMkCK);
  m.up_off = dual ? (int)(((size_t)m.nr * pitch + 127) & ~(size_t)127) : 0;
  return m;
}

size_t mk_scratch_bytes(int H, int I, int qd, int G, int hd, int nsplit) {
  const size_t xs = (size_t)std::max({H, I, qd}) * 4;
  // attention: q heads, new k and v, scores / numerators / rescales of a
  // tile; then, in the CTA merging a kv head, every split's partial
  // (o, max, sum) plus a weight per split and head
  // merge of a slice of one kv head's outputs: (max, sum) per split and
  // head, 1 / sum per head, weighted partials per split and output
  const size_t splits = (size_t)nsplit;
  const size_t slice = ((size_t)G * hd + splits - 1) / splits + 1;
  const size_t att = std::max((size_t)G * hd + 2 * hd + 2 * 32 * G + G,
                              2 * splits * G + G + splits * slice) * 4;
  return (std::max(xs, att) + 127) & ~(size_t)127;
}

size_t mk_smem_bytes(size_t scratch_bytes) {
  const size_t total = kMkScrOff + scratch_bytes + (size_t)kMkS * kMkSlot;
  return total <= 227 * 1024 ? total : 0;
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
