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
//     issuing TMA copies of the weights was measured at half of the HBM
//     bandwidth; cp.async from several warps sustains it. For the K/V
//     history the opposite holds at long lengths: from kMkBulkMinLen
//     positions on, each attention tile is two 1-D bulk copies.)
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
// Only the warps that compute a tile wait for it and release it: in
// projections a group of warps owning one column block per thread computes
// a whole tile while the other groups take the next tiles; in attention each
// warp takes one tile of positions for a pair of query heads (scores, online
// softmax, p v). A consumer first waits until the slot's tag (written by the
// producer once the slot's previous tile was released) names its tile, so
// its parity wait on the full barrier can never match an older phase, and
// the releases of a tile add up to the empty barrier's count.
//
// The quantized block dots (quantize.rs:252-280) are integer dp4a products of
// the weight codes with the input staged as fixed-point byte planes per
// 32-column block, combined in f32 and scaled once per block by the weight
// scale and the block's power-of-two input scale. Cross-CTA data
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
// From this history length on, attention tiles come in by two 1-D bulk
// copies (K, V) instead of 1024 16-byte cp.async pieces: measured on the
// Qwen3-4B shape in Q8_0, 4.55 -> 3.74 ms per token at 32768 positions and
// 2.41 -> 2.37 ms at 4096 (with the pieces, the step time followed the
// number of producer warps, not the ring depth), but 1.916 -> 1.935 ms in
// Q4_0 at 2048, where the pieces stay.
constexpr int kMkBulkMinLen = 3072;
static_assert(kMkS % kMkProducers == 0, "each producer warp owns its own slots");
// Projection inputs are staged as exact fixed-point planes: per 32-column
// block, m = rint(x * 2^(kMkFx - e)) with 2^(e-1) <= max|x| < 2^e, written
// as kMkNP signed base-256 digits (plane p holds digit p of every column), so
// that the block dot with the weight codes is a sum of exact integer dp4a
// products. kMkNP = 3 keeps 23 bits of the block maximum (an input's error
// is at most 2^-23 of the block's largest magnitude, about one f32 rounding
// of that element); each further plane would add 8 bits for 8 more dp4a per
// block, and the dp4a count bounds the projection phases.
constexpr int kMkNP = 3;
constexpr int kMkFx = 8 * kMkNP - 2;           // |m| <= 2^kMkFx
// Words of one staged block: 8 * kMkNP plane words (Q4_0: [word j][plane]
// [low / high nibble columns]; Q8_0: [word j][plane]), then kMkNP Q4_0
// offset corrections; a multiple of 4 words for 16-byte loads.
constexpr int kMkRecW = (9 * kMkNP + 3) & ~3;
constexpr int kMkMiscOff = 256;                // small reductions and flags
static_assert(kMkS * (16 + 4) <= kMkMiscOff, "ring barriers and slot tags precede the misc area");
constexpr int kMkCtaOff = 768;                 // the CTA's plan (MkCta)
constexpr int kMkRedOff = 1024;                // projection row sums, 2048 floats
constexpr int kMkRopeOff = 9216;               // cos | sin of this position's RoPE row
constexpr int kMkScrOff = 9728;                // x / attention scratch, then the ring

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Shared-memory loads by 32-bit shared address: the ring slots and the
// staged inputs are reached through pointers whose address space the
// compiler cannot always see, and a generic load to shared memory takes the
// slower L1 path. Volatile keeps them after the mbarrier waits (also volatile).
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 lds_f32x2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds_f32x4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds_u32x4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}

// 4-way byte dot products with 32-bit accumulate: unsigned codes (Q4_0
// nibbles times 16) or signed codes (Q8_0) against signed plane digits.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Low bytes of four ints packed into one word (a in byte 0).
__device__ __forceinline__ uint32_t pack_lo_bytes(int a, int b, int c, int d) {
  const uint32_t ab = __byte_perm((uint32_t)a, (uint32_t)b, 0x0040);
  const uint32_t cd = __byte_perm((uint32_t)c, (uint32_t)d, 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}

// Block dot of one row block (quantize.rs:252-280: sum over the block of
// code * x, times the scale d) against the staged planes xw of the same
// columns, before the block's power-of-two input scale: exact integer sums
// per plane, combined in f32. Q4_0 codes enter as 16 * nibble; the block's
// -8 offset is the staged correction (-128 * digit sum per plane), which
// also starts each plane's sum.
template <int DT>
__device__ __forceinline__ float mk_block_dot(uint32_t blk, const uint32_t (&xw)[kMkRecW]) {
  const float d = lds_f32(blk);  // blk: shared address of the block
  int s[kMkNP];
  if (DT == MINQ_Q8_0) {
#pragma unroll
    for (int q = 0; q < kMkNP; ++q) s[q] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t w = lds_u32(blk + 4 + 4 * j);
#pragma unroll
      for (int q = 0; q < kMkNP; ++q) s[q] = dp4a_ss(w, xw[j * kMkNP + q], s[q]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < kMkNP; ++q) s[q] = (int)xw[8 * kMkNP + q];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = lds_u32(blk + 4 + 4 * j);
      const uint32_t hi = w & 0xF0F0F0F0u;          // 16 * high nibbles: odd columns
      const uint32_t lo = (w << 4) & 0xF0F0F0F0u;   // 16 * low nibbles: even columns
#pragma unroll
      for (int q = 0; q < kMkNP; ++q) {
        s[q] = dp4a_us(lo, xw[j * 2 * kMkNP + 2 * q], s[q]);
        s[q] = dp4a_us(hi, xw[j * 2 * kMkNP + 2 * q + 1], s[q]);
      }
    }
  }
  // sum_q 256^q s[q] in f32: pairs of planes combine exactly in 32 bits
  float f;
  if (kMkNP == 4) {
    const int hi = s[3] * 256 + s[2], lo = s[1] * 256 + s[0];
    f = fmaf((float)hi, 65536.0f, (float)lo);
  } else {
    f = (float)s[kMkNP - 1];
#pragma unroll
    for (int q = kMkNP - 2; q >= 0; --q) f = fmaf(f, 256.0f, (float)s[q]);
  }
  return f * d;
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

// Rows [rb, rb + cnt) of this CTA in a projection: cnt * nb contiguous
// blocks of the row-major matrix, streamed as tiles of kMkTileBlocks blocks
// (the last one shorter), gate and up tiles alternating in the dual phase.
struct MkShare {
  int rb, cnt;
};
template <int DT>
struct MkTile {
  // blocks per tile: a whole number of blocks and of 16-byte pieces, <= a slot
  static constexpr int blocks = DT == MINQ_Q8_0 ? 452 : 816;
};

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

template <int DT>
__device__ void mk_cta_plan(const MkParams& p, int L, MkCta* c) {
  for (int ph = 0; ph < 5; ++ph) {
    if (ph == 1) continue;
    const MkMat& m = mk_mat(p, ph);
    mk_share(m.rows, &c->sh[ph].rb, &c->sh[ph].cnt);
    const long long blocks = (long long)c->sh[ph].cnt * (m.cols / kBlock);
    c->tiles[ph] = (ph == 3 ? 2 : 1) * (int)((blocks + MkTile<DT>::blocks - 1) / MkTile<DT>::blocks);
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
  const MkLayerPtrs* lps;  // the per-layer pointers, copied to shared memory
  uint64_t* full;   // [kMkS]: the producer lanes' copies of the slot's tile landed
  uint64_t* empty;  // [kMkS]: the warps computing the slot's tile released it
  int* tag;         // [kMkS]: the tile last issued into the slot
  int li, ph, idx;  // next tile to issue: layer, phase, index in the phase
  int issued;       // tiles issued so far (slot = issued % kMkS)
};

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

// Advance the iterator past phases without tiles; false past the last layer.
__device__ __forceinline__ bool mk_feed_settle(const MkParams& p, MkFeed& f, const MkCta* cta) {
  while (f.li < p.n_layers && f.idx >= cta->tiles[f.ph]) {
    f.idx = 0;
    if (++f.ph == 5) {
      f.ph = 0;
      ++f.li;
    }
  }
  return f.li < p.n_layers;
}

// Step the iterator over one tile without copying it.
__device__ __forceinline__ void mk_feed_skip(MkFeed& f) {
  ++f.idx;
  ++f.issued;
}

// Producer warp: copy the current tile into its slot with the warp's 32
// lanes, then have the slot's full barrier track the copies
// (cp.async.mbarrier.arrive). Projection tiles: a contiguous run of the
// CTA's blocks (gate and up alternating in the gate/up phase). Attention
// tiles: the pieces of K (swizzled) and of V, or from kMkBulkMinLen on two
// bulk copies. False on abort.
template <int DT>
__device__ bool mk_issue(const MkParams& p, MkFeed& f, const MkCta* cta, int L) {
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  const int lane = threadIdx.x & 31;
  if (!mk_wait_empty(p, f, f.issued)) return false;
  const int slot = f.issued % kMkS;
  // the slot now takes tile f.issued: its previous tile was computed and
  // released, so a consumer that sees this tag waits on the right phase
  if (lane == 0) st_release_shared(&f.tag[slot], f.issued);
  unsigned char* dst = f.ring + (size_t)slot * kMkSlot;
  const MkLayerPtrs& lp = f.lps[f.li];
  if (f.ph == 1) {
    const int hd = p.hd, tp = 2048 / hd;
    const int p0 = (cta->t0 + f.idx) * tp, np = min(tp, L - p0);
    const size_t off = (size_t)f.li * p.cache_layer_stride + (size_t)cta->kh * p.max_seq * hd +
                       (size_t)p0 * hd;
    if (L >= kMkBulkMinLen) {
      // K and V rows of the tile are contiguous runs of the head-major
      // cache: one 1-D bulk copy each (the TMA engine), completing on the
      // slot's full barrier as transaction bytes; the other lanes arrive
      // without a copy, so the barrier still counts the warp's 32 lanes
      const uint32_t bytes = (uint32_t)(np * hd * 4);
      if (lane == 0) {
        mbar_arrive_expect_tx(&f.full[slot], 2 * bytes);
        bulk_g2s(dst, p.kc + off, bytes, &f.full[slot]);
        bulk_g2s(dst + tp * hd * 4, p.vc + off, bytes, &f.full[slot]);
      } else {
        mbar_arrive(&f.full[slot]);
      }
      mk_feed_skip(f);
      return true;
    }
    // K row r's 16-byte chunk c lands at chunk c ^ (r mod 16) of the row (16
    // <= the chunks per row), so the consumer's lane r reads chunk c of its
    // row where every lane reads chunk c of q without a bank conflict
    const int nch = hd / 4, pieces = np * nch;  // 16-byte pieces of K (and of V)
    for (int i = lane; i < pieces; i += 32) {
      const int r = i / nch, c = i - r * nch;
      cp_async16(dst + (r * nch + (c ^ (r & 15))) * 16, p.kc + off + i * 4);
      cp_async16(dst + tp * hd * 4 + i * 16, p.vc + off + i * 4);
    }
  } else {
    const bool dual = f.ph == 3;
    const MkMat& m = mk_mat(p, f.ph);
    const MkShare& sh = cta->sh[f.ph];
    const int nb = m.cols / kBlock, up = dual ? (f.idx & 1) : 0, k = dual ? f.idx >> 1 : f.idx;
    const uint8_t* w = f.ph == 0 ? lp.w_qkv : f.ph == 2 ? lp.w_o : dual ? (up ? lp.w_up : lp.w_gate)
                                                                         : lp.w_down;
    const long long g0 = (long long)k * MkTile<DT>::blocks;
    const int nblk = (int)min((long long)MkTile<DT>::blocks, (long long)sh.cnt * nb - g0);
    const unsigned char* src = w + ((size_t)sh.rb * nb + (size_t)g0) * BB;
    const int pieces = nblk * BB / 16;  // rows are 16-byte multiples (nb % 4 == 0)
#pragma unroll 4
    for (int i = lane; i < pieces; i += 32) cp_async16(dst + i * 16, src + (size_t)i * 16);
  }
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&f.full[slot]))
               : "memory");
  mk_feed_skip(f);
  return true;
}

// Producer warp k (of kMkProducers) issues the tiles k, k + kMkProducers, ...
// Because kMkS is a multiple of kMkProducers it alone refills those slots.
template <int DT>
__device__ void mk_producer(const MkParams& p, MkFeed& f, const MkCta* cta, int L) {
  const int k = ((int)threadIdx.x - kMkConsumers) >> 5;
  int last[kMkS / kMkProducers];  // the last tile issued into each own slot
#pragma unroll
  for (int j = 0; j < kMkS / kMkProducers; ++j) last[j] = -1;
  if (!*reinterpret_cast<volatile int*>(p.abort_flag)) {
    while (mk_feed_settle(p, f, cta)) {
      if (f.issued % kMkProducers == k) {
        const int it = f.issued;
        if (!mk_issue<DT>(p, f, cta, L)) break;
        last[(it % kMkS) / kMkProducers] = it;
      } else {
        mk_feed_skip(f);
      }
    }
  }
  // nothing in flight at exit (the consumers skip their waits after an
  // abort): this warp's cp.async pieces, then the bulk copies, whose
  // completion is the full phase of the slot's last tile (time-bounded)
  asm volatile("cp.async.wait_all;" ::: "memory");
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int j = 0; j < kMkS / kMkProducers; ++j)
      if (last[j] >= 0)
        mbar_wait_timed(&f.full[last[j] % kMkS], (uint32_t)(last[j] / kMkS) & 1u, p.status);
  }
  __syncwarp();
}

// Consumer wait for the tile `it`; never leaves the caller's barrier
// sequence: after an abort (or its own timeout, which raises the abort) it
// returns at once with stale data, and every CTA stops at the next grid
// barrier.
__device__ const unsigned char* mk_next_tile(const MkParams& p, const MkFeed& f, int it) {
  const int s = it % kMkS;
  const uint32_t parity = (uint32_t)(it / kMkS) & 1u;
  // first the slot's tag: once it names this tile, the slot's previous tile
  // was complete, so the parity wait below cannot match an older phase
  if (ld_acquire_shared(&f.tag[s]) != it) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t n = 1; ld_acquire_shared(&f.tag[s]) != it; ++n) {
      if ((n & 15) == 0) {
        if (*reinterpret_cast<volatile int*>(p.abort_flag)) return f.ring + (size_t)s * kMkSlot;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.status, kDeviceTimeout);
          atomicExch(p.abort_flag, 1);
          return f.ring + (size_t)s * kMkSlot;
        }
      }
    }
  }
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

// The warp is done with tile `it`; the warps computing a tile release it
// with counts that add up to kMkCW.
__device__ __forceinline__ void mk_release(const MkFeed& f, int it, uint32_t count) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_count(&f.empty[it % kMkS], count);
}
// ---------------------------------------------------------------- consumers

__device__ __forceinline__ void mk_sync() { named_barrier_sync(1, kMkConsumers); }

// Grid barrier over the consumers of all CTAs (monotonic 64-bit counter).
__device__ bool mk_grid_sync(const MkParams& p, unsigned long long target, int* flag) {
  mk_sync();
  if (threadIdx.x == 0) {
    // arrival: a release add (the CTA's writes, ordered before by the named
    // barrier, become visible with it), no round trip for a return value
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar_ctr) : "memory");
    int ok = 1;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t n = 1;; ++n) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p.bar_ctr) : "memory");
      if (v >= target) break;
      if ((n & 15) == 0) {  // the abort flag and the time limit, now and then
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
    // no trailing fence: the acquire load that saw the last arrival orders
    // this CTA's later reads after every CTA's released writes, and the named
    // barrier below extends that order to the CTA's other threads
    *reinterpret_cast<volatile int*>(flag) = ok;
  }
  mk_sync();
  return *reinterpret_cast<volatile int*>(flag) != 0;
}

// The residual stream's (value, epoch) pairs (MkParams::xr_*): one 8-byte
// store per row, so a reader never sees a value without its epoch.
__device__ __forceinline__ void mk_st_pair(uint2* dst, float v, unsigned ep) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(dst), "r"(__float_as_uint(v)),
               "r"(ep)
               : "memory");
}
__device__ __forceinline__ uint4 mk_ld_pairs2(const uint2* src) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(src)
               : "memory");
  return v;
}

// Give up a wait: the device status word and the abort flag.
__device__ __forceinline__ bool mk_wait_expired(const MkParams& p, uint64_t t0) {
  if (*reinterpret_cast<volatile int*>(p.abort_flag)) return true;
  if (global_timer_ns() - t0 > kWaitLimitNs) {
    atomicOr(p.status, kDeviceTimeout);
    atomicExch(p.abort_flag, 1);
    return true;
  }
  return false;
}

// x[i .. i + 7] of an exchange site (src = slot 0 at element i, slots H
// apart): every pair of the nsum slots is waited for until it carries epoch
// ep (bounded), then the values are summed over the slots in rank order.
template <int NW>
__device__ __forceinline__ void mk_ld8_site(const MkParams& p, const uint2* src, unsigned ep,
                                            float4& a, float4& b) {
#pragma unroll 1
  for (int q = 0; q < NW; ++q) {
    const uint2* e = src + (size_t)q * p.H;
    uint4 w0 = mk_ld_pairs2(e), w1 = mk_ld_pairs2(e + 2), w2 = mk_ld_pairs2(e + 4),
          w3 = mk_ld_pairs2(e + 6);
    if (((w0.y ^ ep) | (w0.w ^ ep) | (w1.y ^ ep) | (w1.w ^ ep) | (w2.y ^ ep) | (w2.w ^ ep) |
         (w3.y ^ ep) | (w3.w ^ ep)) != 0u) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t n = 1;; ++n) {
        w0 = mk_ld_pairs2(e);
        w1 = mk_ld_pairs2(e + 2);
        w2 = mk_ld_pairs2(e + 4);
        w3 = mk_ld_pairs2(e + 6);
        if (((w0.y ^ ep) | (w0.w ^ ep) | (w1.y ^ ep) | (w1.w ^ ep) | (w2.y ^ ep) | (w2.w ^ ep) |
             (w3.y ^ ep) | (w3.w ^ ep)) == 0u)
          break;
        if ((n & 15) == 0 && mk_wait_expired(p, t0)) break;
        __nanosleep(64);  // fewer polls of L2 while the rows arrive
      }
    }
    const float4 ca = make_float4(__uint_as_float(w0.x), __uint_as_float(w0.z),
                                  __uint_as_float(w1.x), __uint_as_float(w1.z));
    const float4 cb = make_float4(__uint_as_float(w2.x), __uint_as_float(w2.z),
                                  __uint_as_float(w3.x), __uint_as_float(w3.z));
    if (q == 0) {
      a = ca;
      b = cb;
    } else {
      a.x += ca.x; a.y += ca.y; a.z += ca.z; a.w += ca.w;
      b.x += cb.x; b.y += cb.y; b.z += cb.z; b.w += cb.w;
    }
  }
}

// x[i] of an exchange site (src = slot 0 at element i), as mk_ld8_site.
template <int NW>
__device__ __forceinline__ float mk_ld1_site(const MkParams& p, const uint2* src, unsigned ep) {
  float a = 0.0f;
#pragma unroll 1
  for (int q = 0; q < NW; ++q) {
    const uint2* e = src + (size_t)q * p.H;
    uint2 w;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(e) : "memory");
    if (w.y != ep) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t n = 1;; ++n) {
        asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(e) : "memory");
        if (w.y == ep) break;
        if ((n & 15) == 0 && mk_wait_expired(p, t0)) break;
      }
    }
    a = q == 0 ? __uint_as_float(w.x) : a + __uint_as_float(w.x);
  }
  return a;
}

// Stage the lm_head input in shared memory: xs = rmsnorm(src) * gain
// (tensor.rs:219-227), n floats, n % 8 == 0; src is the last exchange site.
template <int NW>
__device__ void mk_stage_x(const MkParams& p, float* xs, const float* x, const uint2* site,
                           unsigned ep, int n, const float* gain, float* misc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = n >> 3;
  float4* xs4 = reinterpret_cast<float4*>(xs);
  float ss = 0.0f;
  for (int gi = tid; gi < ng; gi += kMkConsumers) {
    float4 a, b;
    if constexpr (NW == 1) {
      a = ldcg4(x + 8 * gi);
      b = ldcg4(x + 8 * gi + 4);
    } else {
      mk_ld8_site<NW>(p, site + 8 * gi, ep, a, b);
    }
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
  const float inv = 1.0f / sqrtf(v / (float)n + p.eps);
  const float4* g4 = reinterpret_cast<const float4*>(gain);
  for (int gi = tid; gi < ng; gi += kMkConsumers) {
    float4 a = xs4[2 * gi], b = xs4[2 * gi + 1];
    const float4 ga = g4[2 * gi], gb = g4[2 * gi + 1];
    a.x = a.x * inv * ga.x; a.y = a.y * inv * ga.y; a.z = a.z * inv * ga.z; a.w = a.w * inv * ga.w;
    b.x = b.x * inv * gb.x; b.y = b.y * inv * gb.y; b.z = b.z * inv * gb.z; b.w = b.w * inv * gb.w;
    xs4[2 * gi] = a;
    xs4[2 * gi + 1] = b;
  }
  mk_sync();
}

// Stage a projection input as fixed-point planes: v = src (n floats, n % 32
// == 0), or, with `site`, the residual stream of an exchange site (the sum
// of its nsum slots once they carry epoch ep), times gain when gain is set,
// then per 32-column block b:
// e = exponent of max|v| (2^(e-1) <= max < 2^e), m = rint(v * 2^(kMkFx - e))
// (|m| <= 2^kMkFx), split into kMkNP signed base-256 digits
// (m = sum_q 256^q d_q, d_q in [-128, 127]). xp gets kMkRecW words per block
// (see mk_block_dot for their order) and xsb the block's scale 2^(e - kMkFx)
// (over 16 for Q4_0, whose codes enter as 16 * nibble). Thread t stages the 8
// columns 8 (t mod 4) .. + 7 of block t / 4, so the four threads of a block
// are adjacent lanes. With a gain, warp w also leaves its part of sum(src^2)
// in misc[w]: RMSNorm (tensor.rs:219-227) is linear in the input, so its
// scale 1 / rms multiplies each row's sum in the projection's epilogue and
// the planes need not wait for the reduction.
template <int DT, int NW>
__device__ void mk_stage_planes(const MkParams& p, uint32_t* xp, float* xsb, const float* src,
                                const uint2* site, unsigned ep, int n, const float* gain,
                                float* misc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = n >> 3;
  const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  // every load first (n <= 16384: at most four rounds of 512 groups of 8)
  constexpr int MR = 4;
  float4 va[MR], vb[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    const int gi = tid + r * kMkConsumers;
    if (gi >= ng) {
      va[r] = zero;
      vb[r] = zero;
    } else if (NW > 1 && site) {
      mk_ld8_site<NW>(p, site + 8 * gi, ep, va[r], vb[r]);
    } else {
      va[r] = ldcg4(src + 8 * gi);
      vb[r] = ldcg4(src + 8 * gi + 4);
    }
  }
  if (gain) {
    float ss = 0.0f;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      const float4 a = va[r], b = vb[r];
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
    if (lane == 0) misc[warp] = ss;  // read after the closing barrier
  }
  const float4* g4 = reinterpret_cast<const float4*>(gain);
#pragma unroll
  for (int rd = 0; rd < MR; ++rd) {
    if (rd * kMkConsumers >= ng) break;  // the same for every thread
    const int gi = tid + rd * kMkConsumers;
    const bool act = gi < ng;
    float4 a = va[rd], b = vb[rd];
    if (gain && act) {
      const float4 ga = g4[2 * gi], gb = g4[2 * gi + 1];
      a.x *= ga.x; a.y *= ga.y; a.z *= ga.z; a.w *= ga.w;
      b.x *= gb.x; b.y *= gb.y; b.z *= gb.z; b.w *= gb.w;
    }
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    // e from the exponent field; tiny blocks (< 2^-91) clamp to e = -90
    const int e = max((int)((__float_as_uint(mx) >> 23) & 0xFFu) - 126, -90);
    const float scale = __uint_as_float((uint32_t)(127 + kMkFx - e) << 23);  // 2^(kMkFx - e)
    int r[kMkNP][8];   // r[0] = m, r[q+1] = floor((r[q] + 128) / 256); digit q = low byte of r[q]
    int dsum[kMkNP];   // sum of the digits d_q = r[q] - 256 r[q+1] (last: r[q])
#pragma unroll
    for (int q = 0; q < kMkNP; ++q) dsum[q] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r[0][i] = __float2int_rn(v[i] * scale);
#pragma unroll
      for (int q = 1; q < kMkNP; ++q) r[q][i] = (r[q - 1][i] + 128) >> 8;
#pragma unroll
      for (int q = 0; q < kMkNP; ++q)
        dsum[q] += q + 1 < kMkNP ? r[q][i] - 256 * r[q + 1][i] : r[q][i];
    }
    uint32_t w[2 * kMkNP];
#pragma unroll
    for (int q = 0; q < kMkNP; ++q) {
      if (DT == MINQ_Q4_0) {  // word j = t mod 4: even columns (low nibbles), odd (high)
        w[2 * q] = pack_lo_bytes(r[q][0], r[q][2], r[q][4], r[q][6]);
        w[2 * q + 1] = pack_lo_bytes(r[q][1], r[q][3], r[q][5], r[q][7]);
      } else {                // words 2 (t mod 4) and 2 (t mod 4) + 1, plane-minor
        w[q] = pack_lo_bytes(r[q][0], r[q][1], r[q][2], r[q][3]);
        w[kMkNP + q] = pack_lo_bytes(r[q][4], r[q][5], r[q][6], r[q][7]);
      }
    }
#pragma unroll
    for (int q = 0; q < kMkNP; ++q) {
      dsum[q] += __shfl_xor_sync(0xffffffffu, dsum[q], 1);
      dsum[q] += __shfl_xor_sync(0xffffffffu, dsum[q], 2);
    }
    if (act) {
      uint32_t* rec = xp + (size_t)(gi >> 2) * kMkRecW;
      uint2* dst = reinterpret_cast<uint2*>(rec + (gi & 3) * 2 * kMkNP);
#pragma unroll
      for (int q = 0; q < kMkNP; ++q) dst[q] = make_uint2(w[2 * q], w[2 * q + 1]);
      if ((gi & 3) == 0) {
#pragma unroll
        for (int q = 0; q < kMkNP; ++q)
          rec[8 * kMkNP + q] = DT == MINQ_Q4_0 ? (uint32_t)(-128 * dsum[q]) : 0u;
        xsb[gi >> 2] = __uint_as_float((uint32_t)(127 + e - kMkFx - (DT == MINQ_Q4_0 ? 4 : 0)) << 23);
      }
    }
  }
  mk_sync();
}

// One projection phase over the CTA's rows [rb, rb + cnt). Every consumer
// thread owns one column block for the whole phase: warps form T = 16 / WG
// groups of WG = ceil(nb / 32) (nb blocks per row), warp wc of a group takes
// blocks 32 wc + lane, and its staged input planes stay in registers. Group
// r processes the tiles tt = r mod T (a tile is a run of the CTA's row-major
// blocks), so T tiles are in work at once; for each row of its tile a warp
// sums its lanes' block dots and writes red[tile parity][half][row][wc] (a
// row spans at most two tiles, which differ in parity: one writer per
// entry). epi(row, v0, v1, pre) (v1 = up for the dual gate/up form) gets
// the rows summed over parity and wc in a fixed order, and pre = pre_ld(row),
// loaded when the phase starts (thread t < cnt takes row rb + t).
template <int DT, bool DUAL, class Pre, class Epi>
__device__ void mk_consume_mat(const MkParams& p, const MkMat& m, const uint32_t* xp,
                               const float* xsb, MkFeed& f, const MkCta* cta, int L, float* red,
                               int& it, const float* norm_ss, int norm_n, Pre pre_ld, Epi epi) {
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  constexpr int TB = MkTile<DT>::blocks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = m.cols / kBlock, WG = (nb + 31) >> 5, T = kMkCW / WG;
  const int grp = warp / WG, wc = warp - grp * WG, col = 32 * wc + lane;
  const bool in_grp = grp < T, has_col = in_grp && col < nb;
  int rb, cnt;
  mk_share(m.rows, &rb, &cnt);
  const int halves = DUAL ? 2 : 1;
  // this thread's column: staged planes and scale, kept for the phase
  uint32_t xw[kMkRecW];
  float sb = 0.0f;
  {
    const uint32_t rec = smem_u32(xp) + (uint32_t)(has_col ? col : 0) * kMkRecW * 4;
#pragma unroll
    for (int i = 0; i < kMkRecW / 4; ++i) {
      const uint4 v = lds_u32x4(rec + 16 * i);
      xw[4 * i] = v.x;
      xw[4 * i + 1] = v.y;
      xw[4 * i + 2] = v.z;
      xw[4 * i + 3] = v.w;
    }
    if (has_col) sb = xsb[col];
  }
  const float pre = tid < cnt ? pre_ld(rb + tid) : 0.0f;  // cnt <= 512
  const int plane = halves * cnt * WG;  // floats per tile parity
  for (int i = tid; i < 2 * plane; i += kMkConsumers) red[i] = 0.0f;
  mk_sync();
  const int total = cnt * nb;  // < 2^16 for every eligible shape
  const int per = (total + TB - 1) / TB;  // tiles per matrix
  // tile tt of the phase at `tile`, computed by this warp's group
  auto work = [&](const unsigned char* tile, int tt) {
    const int half = DUAL ? (tt & 1) : 0, k = DUAL ? tt >> 1 : tt;
    const int g0 = k * TB, g1 = min(g0 + TB, total);
    const int r_lo = g0 / nb, r_hi = (g1 - 1) / nb;
    float* rr = red + (k & 1) * plane + half * cnt * WG + wc;
    const uint32_t base = smem_u32(tile) - (uint32_t)(g0 * BB);  // block g at base + g * BB
    for (int R = r_lo; R <= r_hi; R += 4) {  // four rows at a time for ILP
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int g = (R + k) * nb + col;
        v[k] = col < nb && R + k <= r_hi && g >= g0 && g < g1
                   ? mk_block_dot<DT>(base + (uint32_t)(g * BB), xw) * sb
                   : 0.0f;
      }
      // transposed warp sum of the four rows: the upper half-warp keeps
      // rows 2, 3 and sends rows 0, 1, then lanes with bit 3 set keep the
      // odd row; the lanes 0, 8, 16, 24 end with rows R .. R + 3
      const bool u16 = lane & 16, u8 = lane & 8;
      float a0 = u16 ? v[2] : v[0], a1 = u16 ? v[3] : v[1];
      a0 += __shfl_xor_sync(0xffffffffu, u16 ? v[0] : v[2], 16);
      a1 += __shfl_xor_sync(0xffffffffu, u16 ? v[1] : v[3], 16);
      float s = u8 ? a1 : a0;
      s += __shfl_xor_sync(0xffffffffu, u8 ? a0 : a1, 8);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      const int k = ((lane >> 4) << 1) | ((lane >> 3) & 1);
      if ((lane & 7) == 0 && R + k <= r_hi) rr[(size_t)(R + k) * WG] = s;
    }
  };
  // Group g computes the tiles g, g + T, ...: its warps wait only for those
  // (tag, then full barrier) and release them with counts adding up to
  // kMkCW; the other warps never touch them.
  const int ntl = halves * per;
  if (in_grp) {
    const uint32_t cnt_rel = wc == 0 ? (uint32_t)(kMkCW - WG + 1) : 1u;
    for (int tt = grp; tt < ntl; tt += T) {
      work(mk_next_tile(p, f, it + tt), tt);
      mk_release(f, it + tt, cnt_rel);
    }
  }
  it += ntl;
  mk_sync();
  if (tid < cnt) {
    const int t = tid;
    float v0 = 0.0f, v1 = 0.0f;
    for (int q = 0; q < 2; ++q)
      for (int w = 0; w < WG; ++w) {
        v0 += red[q * plane + (size_t)t * WG + w];
        if (DUAL) v1 += red[q * plane + ((size_t)cnt + t) * WG + w];
      }
    if (norm_ss) {  // the RMSNorm scale of the staged input (mk_stage_planes)
      float ss = 0.0f;
#pragma unroll
      for (int w = 0; w < kMkCW; ++w) ss += norm_ss[w];
      const float inv = 1.0f / sqrtf(ss / (float)norm_n + p.eps);
      v0 *= inv;
      v1 *= inv;
    }
    epi(rb + t, v0, v1, pre);
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

// One tile of the online softmax of a pair of query heads of the kv head,
// run by one warp (model.rs:223-248: s = q.k / sqrt(hd), softmax over
// positions, o = sum p v). Lane l owns dims DPL l .. DPL l + DPL - 1 and
// keeps those of both heads' queries in registers (q); for 16 positions at a
// time it forms the partial products with each K row, and one transposed
// warp sum of the 32 partials (16 positions x 2 heads) leaves lane l with
// the score of position l mod 16 for head l / 16. The running max m and sum
// l are replicated in every lane, o[g] holds the lane's dims of head g; only
// heads g < gw are live. Ks: K rows in the producer's swizzled chunk order
// (swz: the cp.async tiles) or plain (bulk-copied tiles, the new position);
// V: plain rows. np >= 1 positions.
template <int DPL>
__device__ __forceinline__ void mk_attn_tile(const float (&q)[2][DPL], int gw, uint32_t Ks,
                                             bool swz, uint32_t V, int np, float scale,
                                             float (&m)[2], float (&l)[2], float (&o)[2][DPL]) {
  constexpr int HD = 32 * DPL;
  const int lane = threadIdx.x & 31, hl = lane >> 4, jl = lane & 15;
  for (int j0 = 0; j0 < np; j0 += 16) {
    float v[32];  // v[16 g + j]: this lane's partial of head g at position j0 + j
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float k[DPL];
#pragma unroll
      for (int e = 0; e < DPL; ++e) k[e] = 0.0f;
      const int jj = j0 + j;
      if (jj < np) {
        const int sw = swz ? (jj & 15) : 0;
        const uint32_t row = Ks + (uint32_t)(jj * HD * 4);
        if constexpr (DPL == 4) {
          const float4 k4 = lds_f32x4(row + (uint32_t)(16 * (lane ^ sw)));
          k[0] = k4.x;
          k[1] = k4.y;
          k[2] = k4.z;
          k[3] = k4.w;
        } else {
          const float2 k2 = lds_f32x2(row + (uint32_t)(16 * ((lane >> 1) ^ sw) + 8 * (lane & 1)));
          k[0] = k2.x;
          k[1] = k2.y;
        }
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) a = fmaf(q[g][e], k[e], a);
        v[16 * g + j] = a;
      }
    }
    // transposed warp sum: at the level of lane bit b the lanes with bit b
    // set keep the upper half of their values and send the lower half
#pragma unroll
    for (int lv = 0; lv < 5; ++lv) {
      const int b = 16 >> lv, n = 16 >> lv;
      const bool up = (lane & b) != 0;
#pragma unroll
      for (int i = 0; i < n; ++i) {
        const float keep = up ? v[i + n] : v[i], send = up ? v[i] : v[i + n];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, b);
      }
    }
    const bool valid = j0 + jl < np && hl < gw;
    const float sc = valid ? v[0] * scale : -INFINITY;
    float mt = sc;  // tile max of head hl over the 16 lanes of its half-warp
#pragma unroll
    for (int o_ = 8; o_ > 0; o_ >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o_));
    const float mtg[2] = {__shfl_sync(0xffffffffu, mt, 0), __shfl_sync(0xffffffffu, mt, 16)};
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const float mn = fmaxf(m[g], mtg[g]);
      const float c = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
      m[g] = mn;
      l[g] *= c;
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[g][e] *= c;
    }
    const float pr = valid ? expf(sc - (hl ? m[1] : m[0])) : 0.0f;
    float ps = pr;
#pragma unroll
    for (int o_ = 8; o_ > 0; o_ >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o_);
    l[0] += __shfl_sync(0xffffffffu, ps, 0);
    l[1] += __shfl_sync(0xffffffffu, ps, 16);
    const int nj = min(16, np - j0);
#pragma unroll 4
    for (int j = 0; j < nj; ++j) {
      const uint32_t vr = V + (uint32_t)(((j0 + j) * HD + DPL * lane) * 4);
      float vv[DPL];
      if constexpr (DPL == 4) {
        const float4 v4 = lds_f32x4(vr);
        vv[0] = v4.x;
        vv[1] = v4.y;
        vv[2] = v4.z;
        vv[3] = v4.w;
      } else {
        const float2 v2 = lds_f32x2(vr);
        vv[0] = v2.x;
        vv[1] = v2.y;
      }
      const float p0 = __shfl_sync(0xffffffffu, pr, j), p1 = __shfl_sync(0xffffffffu, pr, 16 + j);
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        o[0][e] = fmaf(p0, vv[e], o[0][e]);
        o[1][e] = fmaf(p1, vv[e], o[1][e]);
      }
    }
  }
}

// Attention phase of one CTA: kv head kh, history tiles [t0, t1) of TP
// positions (K rows, swizzled below kMkBulkMinLen, then V rows, in the
// slot) and, in the head's last split, the new position. The query heads form HG = ceil(G / 2) pairs;
// warp w serves pair w mod HG on the tiles t0 + w / HG, t0 + w / HG + 16 / HG,
// ..., the new position going to the warps next in that order; the warp
// states then merge
// into this split's partial (o, m, l) per head. The last split of the
// head to arrive (a counter per head) merges all of the head's split
// partials into the attention output; the others go on to the grid barrier.
template <int DT, int DPL>
__device__ void mk_consume_attn(const MkParams& p, int li, int L, unsigned hbase, float* scr,
                                MkFeed& f, const MkCta* cta, const float* rope_cs, int* misc_i,
                                int& it) {
  int kh, t0, t1;
  bool last;
  if (!mk_attn_item(p, L, &kh, &t0, &t1, &last)) return;
  constexpr int HD = 32 * DPL, TP = 2048 / HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int HPW = 2;  // query heads per warp
  const int G = p.G, HG = (G + HPW - 1) / HPW, WPG = kMkCW / HG;
  const int g0 = (warp % HG) * HPW, gw = min(HPW, G - g0), slot = warp / HG;
  const bool served = warp < HG * WPG;
  float* qs = scr;                     // [G][hd] RoPE'd (and normed) query heads
  float* knew = qs + G * HD;           // [hd] the new position's key (last split)
  float* vnew = knew + HD;             // [hd]
  float* wst = vnew + HD;              // [16][HPW][hd + 2] per-warp o, m, l
  float* fw = wst + kMkCW * HPW * (HD + 2);  // merge: weights and the splits' partials
  const MkLayerPtrs& lp = f.lps[li];
  const size_t head_off = (size_t)li * p.cache_layer_stride + (size_t)kh * p.max_seq * HD;
  // q heads (q_norm, RoPE at position L); the last split also builds the new
  // k (k_norm, RoPE) and v and appends them to the cache
  if (warp < G) {
    mk_head_prep(p, p.qkv_out + (size_t)(kh * G + warp) * HD, lp.q_norm, true, rope_cs,
                 qs + warp * HD);
  } else if (last && warp == G) {
    mk_head_prep(p, p.qkv_out + p.qd + (size_t)kh * HD, lp.k_norm, true, rope_cs, knew);
    __syncwarp();
    for (int i = lane; i < HD; i += 32) p.kc[head_off + (size_t)L * HD + i] = knew[i];
  } else if (last && warp == G + 1) {
    for (int i = lane; i < HD; i += 32) {
      const float v = ldcg(p.qkv_out + p.qd + p.kvd + (size_t)kh * HD + i);
      vnew[i] = v;
      p.vc[head_off + (size_t)L * HD + i] = v;
    }
  }
  mk_sync();
  float m[HPW], l[HPW], o[HPW][DPL];
#pragma unroll
  for (int g = 0; g < HPW; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[g][e] = 0.0f;
  }
  // this warp's two query heads, its lane's dims, in registers
  float q[HPW][DPL];
#pragma unroll
  for (int g = 0; g < HPW; ++g)
#pragma unroll
    for (int e = 0; e < DPL; ++e)
      q[g][e] = served && g < gw ? qs[(g0 + g) * HD + DPL * lane + e] : 0.0f;
  // A tile is computed by the HG warps of its slot (one per head pair):
  // they alone wait for it (tag, then full barrier) and release it, the
  // pair-0 warp with the count that brings the releases to kMkCW.
  const int ntile = t1 - t0;
  if (served) {
    const uint32_t cnt_rel = warp % HG == 0 ? (uint32_t)(kMkCW - HG + 1) : 1u;
    for (int i = slot; i < ntile; i += WPG) {
      const uint32_t kt = smem_u32(mk_next_tile(p, f, it + i));
      mk_attn_tile<DPL>(q, gw, kt, L < kMkBulkMinLen, kt + (uint32_t)(TP * HD * 4),
                        min(TP, L - (t0 + i) * TP), p.scale, m, l, o);
      mk_release(f, it + i, cnt_rel);
    }
  }
  it += ntile;
  if (served && last && ntile % WPG == slot)
    mk_attn_tile<DPL>(q, gw, smem_u32(knew), false, smem_u32(vnew), 1, p.scale, m, l, o);
#pragma unroll
  for (int g = 0; g < HPW; ++g) {
    if (served && g < gw) {
      float* w = wst + (warp * HPW + g) * (HD + 2);
#pragma unroll
      for (int e = 0; e < DPL; ++e) w[DPL * lane + e] = o[g][e];
      if (lane == 0) {
        w[HD] = m[g];
        w[HD + 1] = l[g];
      }
    }
  }
  mk_sync();
  // this split's partial: unnormalised o, max m and sum l per head
  float* part = p.part + (size_t)blockIdx.x * G * (HD + 2);  // [G][hd + 2]
  for (int idx = tid; idx < G * HD; idx += kMkConsumers) {
    const int g = idx / HD, d = idx - g * HD;
    const int wg = g / HPW, gl = g - HPW * wg;  // warps wg, wg + HG, ... hold head g as gl
    float M = -INFINITY;
    for (int w = wg; w < HG * WPG; w += HG) M = fmaxf(M, wst[(w * HPW + gl) * (HD + 2) + HD]);
    float O = 0.0f, Ls = 0.0f;
    for (int w = wg; w < HG * WPG; w += HG) {
      const float* ws = wst + (w * HPW + gl) * (HD + 2);
      const float mw = ws[HD];
      if (mw == -INFINITY) continue;
      const float fr = expf(mw - M);
      O = fmaf(fr, ws[d], O);
      Ls = fmaf(fr, ws[HD + 1], Ls);
    }
    part[g * (HD + 2) + d] = O;
    if (d == 0) {
      part[g * (HD + 2) + HD] = M;
      part[g * (HD + 2) + HD + 1] = Ls;
    }
  }
  // arrival at the head's counter: a release add once the CTA's partial is
  // written (the named barrier orders every thread's writes before it);
  // then every split of the head waits for the head's other splits
  // (bounded) and merges its own slice of the head's outputs
  const int ns = mk_nsplit(p, L);
  mk_sync();
  if (tid == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.head_ctr + kh) : "memory");
    const unsigned target = hbase + (unsigned)(li + 1) * (unsigned)ns;
    int ok = 1;
    const uint64_t tw = global_timer_ns();
    for (uint32_t n = 1;; ++n) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.head_ctr + kh) : "memory");
      if ((int)(v - target) >= 0) break;
      if ((n & 15) == 0) {
        if (*reinterpret_cast<volatile int*>(p.abort_flag)) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - tw > kWaitLimitNs) {
          atomicOr(p.status, kDeviceTimeout);
          atomicExch(p.abort_flag, 1);
          ok = 0;
          break;
        }
      }
    }
    misc_i[2] = ok;
  }
  mk_sync();
  if (!misc_i[2]) return;  // aborting: the launch reports the error
  // split sp merges outputs [o0, o1) of the head (o = g * hd + d): every
  // split's (m, l, o) of them into shared memory in one round of loads,
  // then per output the softmax weights of the splits and the sum
  const int sp = blockIdx.x - kh * ns, no = G * HD;
  const int o0 = (int)((long long)no * sp / ns), o1 = (int)((long long)no * (sp + 1) / ns);
  const int n_o = o1 - o0;
  const float* hp = p.part + (size_t)kh * ns * G * (HD + 2);
  float* sm_m = fw;               // [ns][n_o] each
  float* sm_l = sm_m + ns * n_o;
  float* sm_o = sm_l + ns * n_o;
  for (int i = tid; i < ns * n_o; i += kMkConsumers) {
    const int s_ = i / n_o, j = i - s_ * n_o, od = o0 + j, g = od / HD, d = od - g * HD;
    const float* e = hp + ((size_t)s_ * G + g) * (HD + 2);
    sm_m[i] = __ldcg(e + HD);
    sm_l[i] = __ldcg(e + HD + 1);
    sm_o[i] = __ldcg(e + d);
  }
  mk_sync();
  for (int j = tid; j < n_o; j += kMkConsumers) {
    float M = -INFINITY;
    for (int s_ = 0; s_ < ns; ++s_) M = fmaxf(M, sm_m[s_ * n_o + j]);
    float Ls = 0.0f, O = 0.0f;
    for (int s_ = 0; s_ < ns; ++s_) {
      const float mw = sm_m[s_ * n_o + j];
      const float fs = mw == -INFINITY ? 0.0f : expf(mw - M);
      Ls = fmaf(sm_l[s_ * n_o + j], fs, Ls);
      O = fmaf(sm_o[s_ * n_o + j], fs, O);
    }
    p.att[(size_t)kh * no + o0 + j] = O * (1.0f / Ls);
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

template <int DT, int NW>
__device__ void mk_consumers(const MkParams& p, unsigned char* sm, MkFeed& f, const MkCta* cta,
                             int L, uint32_t tok, unsigned long long bbase, unsigned hbase,
                             unsigned ep) {
  float* misc = reinterpret_cast<float*>(sm + kMkMiscOff);         // [0..32]: reductions
  int* misc_i = reinterpret_cast<int*>(sm + kMkMiscOff + 160);     // flags
  unsigned long long* best_s = reinterpret_cast<unsigned long long*>(sm + kMkMiscOff + 256);
  float* red = reinterpret_cast<float*>(sm + kMkRedOff);
  float* xs = reinterpret_cast<float*>(sm + kMkScrOff);  // attention scratch / lm_head input
  uint32_t* xp = reinterpret_cast<uint32_t*>(sm + kMkScrOff);  // staged projection input
  float* xsb = reinterpret_cast<float*>(xp + (size_t)(max(max(p.H, p.I), p.qd) >> 5) * kMkRecW);
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
  // One GPU (NW == 1): x in p.x, a grid barrier after every phase. Tensor
  // parallel (NW ranks): x in the exchange sites (see MkParams), whose
  // epochs order o_proj / down_proj and their readers instead of a barrier
  // (a barrier across GPUs costs system-scope fences and remote atomics).
  const uint2* xsite = nullptr;  // tensor parallel: the residual stream's site (null: embedding)
  auto site_of = [&](int st) { return p.xr_local + (size_t)st * NW * p.H; };
  auto x_store = [&](int st, int row, float v) {
    const size_t off = ((size_t)st * NW + p.tp_rank) * p.H + row;
#pragma unroll
    for (int q = 0; q < NW; ++q) mk_st_pair(p.xr_dst[q] + off, v, ep);
  };
  const bool add_res = NW == 1 || p.tp_rank == 0;
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const MkLayerPtrs& lp = f.lps[li];
    // P1: q|k|v
    mk_stage_planes<DT, NW>(p, xp, xsb, xsrc, xsite, ep, p.H, lp.attn_norm, misc);
    const float* bias = lp.bias_qkv;
    mk_consume_mat<DT, false>(
        p, p.qkv, xp, xsb, f, cta, L, red, it, misc, p.H,
        [&](int row) { return bias ? bias[row] : 0.0f; },
        [&](int row, float v, float, float b) { p.qkv_out[row] = bias ? v + b : v; });
    if (!(ok = barrier())) break;
    // P2: attention
    if (p.hd == 128) mk_consume_attn<DT, 4>(p, li, L, hbase, xs, f, cta, rope_cs, misc_i, it);
    else mk_consume_attn<DT, 2>(p, li, L, hbase, xs, f, cta, rope_cs, misc_i, it);
    if (!(ok = barrier())) break;
    // P3: x = x + W_o att (tensor parallel: this rank's partial sum, the
    // residual from rank 0 only, into site 2 li of every rank)
    mk_stage_planes<DT, 1>(p, xp, xsb, p.att, nullptr, ep, p.qd, nullptr, misc);
    const uint2* rsite = xsite;
    const float* rsrc = xsrc;
    mk_consume_mat<DT, false>(
        p, p.o, xp, xsb, f, cta, L, red, it, nullptr, 0,
        [&](int row) {
          if constexpr (NW == 1) return ldcg(rsrc + row);
          else {
            if (!add_res) return 0.0f;
            return rsite ? mk_ld1_site<NW>(p, rsite + row, ep) : ldcg(rsrc + row);
          }
        },
        [&](int row, float v, float, float r) {
          if constexpr (NW == 1) p.x[row] = r + v;
          else x_store(2 * li, row, r + v);
        });
    const uint2* xo = NW == 1 ? nullptr : site_of(2 * li);
    if constexpr (NW == 1) {
      xsrc = p.x;
      if (!(ok = barrier())) break;
    }
    // P4: h = silu(gate) * up
    mk_stage_planes<DT, NW>(p, xp, xsb, p.x, xo, ep, p.H, lp.ffn_norm, misc);
    mk_consume_mat<DT, true>(
        p, p.gu, xp, xsb, f, cta, L, red, it, misc, p.H, [&](int) { return 0.0f; },
        [&](int row, float g, float u, float) { p.h[row] = silu(g) * u; });
    if (!(ok = barrier())) break;
    // P5: x = x + W_down h (tensor parallel: into site 2 li + 1)
    mk_stage_planes<DT, 1>(p, xp, xsb, p.h, nullptr, ep, p.I, nullptr, misc);
    mk_consume_mat<DT, false>(
        p, p.down, xp, xsb, f, cta, L, red, it, nullptr, 0,
        [&](int row) {
          if constexpr (NW == 1) return ldcg(p.x + row);
          else return add_res ? mk_ld1_site<NW>(p, xo + row, ep) : 0.0f;
        },
        [&](int row, float v, float, float r) {
          if constexpr (NW == 1) p.x[row] = r + v;
          else x_store(2 * li + 1, row, r + v);
        });
    if constexpr (NW == 1) {
      if (!(ok = barrier())) break;
    } else {
      xsite = site_of(2 * li + 1);
      ok = !*reinterpret_cast<volatile int*>(p.abort_flag);
    }
  }
  if (ok && p.want_logits) {
    mk_stage_x<NW>(p, xs, p.x, xsite, ep, p.H, p.final_norm, misc);
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
  if (NW > 1 && ok && blockIdx.x == 0 && threadIdx.x == 0) *p.xr_epoch = ep;
  if (ok && blockIdx.x == 0 && threadIdx.x == 0) {
    *p.d_pos = L + 1;
    *p.bar_base = bbase + (unsigned long long)nbar * G;
    *p.head_base = hbase + (unsigned)p.n_layers * (unsigned)mk_nsplit(p, L);
  }
}

template <int DT, int NW>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkParams p) {
  extern __shared__ __align__(128) unsigned char sm[];
  const int L = *reinterpret_cast<volatile const int*>(p.d_pos);
  const uint32_t tok = *reinterpret_cast<volatile const uint32_t*>(p.d_tok);
  const unsigned long long bbase = *reinterpret_cast<volatile const unsigned long long*>(p.bar_base);
  const unsigned hbase = *reinterpret_cast<volatile const unsigned*>(p.head_base);
  const unsigned ep = NW > 1 ? *reinterpret_cast<volatile const unsigned*>(p.xr_epoch) + 1u : 0u;
  MkCta* cta = reinterpret_cast<MkCta*>(sm + kMkCtaOff);
  if (threadIdx.x == 0) mk_cta_plan<DT>(p, L, cta);
  __syncthreads();
  MkFeed f;
  f.ring = sm + kMkScrOff + (size_t)p.scratch_bytes;
  // the per-layer pointers after the ring (one copy for the launch)
  MkLayerPtrs* lps = reinterpret_cast<MkLayerPtrs*>(f.ring + (size_t)kMkS * kMkSlot);
  {
    const uint64_t* src = reinterpret_cast<const uint64_t*>(p.layers);
    uint64_t* dst = reinterpret_cast<uint64_t*>(lps);
    const int words = p.n_layers * (int)(sizeof(MkLayerPtrs) / 8);
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  f.lps = lps;
  f.full = reinterpret_cast<uint64_t*>(sm);
  f.empty = f.full + kMkS;
  f.tag = reinterpret_cast<int*>(f.empty + kMkS);
  f.li = 0;
  f.ph = 0;
  f.idx = 0;
  f.issued = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkS; ++s) {
      mbar_init(&f.full[s], 32);     // the issuing producer warp's lanes (cp.async.mbarrier.arrive)
      mbar_init(&f.empty[s], kMkCW);  // kMkCW counts from the warps that compute the tile
      f.tag[s] = -1;
    }
    mbar_fence_init();
  }
  __syncthreads();
  if ((int)threadIdx.x >= kMkConsumers) {
    mk_producer<DT>(p, f, cta, L);
    return;
  }
  mk_consumers<DT, NW>(p, sm, f, cta, L, tok, bbase, hbase, ep);
}

// ---------------------------------------------------------------- host

MkMat mk_plan_mat(int dtype, bool dual, uint64_t rows, uint64_t cols, int grid) {
  const uint64_t nb = cols / kBlock, wg = (nb + 31) / 32, rmax = (rows + grid - 1) / grid;
  const uint64_t tile = dtype == MINQ_Q8_0 ? MkTile<MINQ_Q8_0>::blocks : MkTile<MINQ_Q4_0>::blocks;
  MkMat m{};
  // a row must span at most two tiles (the consumer's row sums by tile parity)
  if (nb == 0 || nb > tile || wg > (uint64_t)kMkCW || 2 * (dual ? 2 : 1) * rmax * wg > 2048 ||
      rmax * nb >= (1u << 16) || rmax > (uint64_t)kMkConsumers)
    return m;
  m.rows = (int)rows;
  m.cols = (int)cols;
  return m;
}

size_t mk_scratch_bytes(int H, int I, int qd, int G, int hd, int nsplit) {
  // staged projection input (planes + one scale per block), or the lm_head input
  const size_t xs = std::max((size_t)(std::max({H, I, qd}) / kBlock) * (kMkRecW * 4 + 4),
                             (size_t)H * 4);
  // attention: q heads, new k and v, the 16 warps' (o, m, l), then the
  // merge's (m, l, o) of every split for this split's slice of the head's
  // G * hd outputs (ns * ceil(G * hd / ns) <= G * hd + ns of each)
  const size_t att = ((size_t)G * hd + 2 * hd + (size_t)kMkCW * 2 * (hd + 2) +
                      3 * ((size_t)G * hd + nsplit)) * 4;
  return (std::max(xs, att) + 127) & ~(size_t)127;
}

size_t mk_smem_bytes(size_t scratch_bytes, int n_layers) {
  const size_t total = kMkScrOff + scratch_bytes + (size_t)kMkS * kMkSlot +
                       (size_t)n_layers * sizeof(MkLayerPtrs);
  return total <= 227 * 1024 ? total : 0;
}

template <int DT, int NW>
static minq_status mk_launch_inst(const MkParams& p, int grid, size_t smem, cudaStream_t s) {
  auto k = decode_mk_kernel<DT, NW>;
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
  count_launch();
  MINQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, p));
  MINQ_LAUNCH_CHECK("decode_mk_kernel");
  return MINQ_OK;
}

minq_status launch_decode_mk(const MkParams& p, int dtype, int grid, size_t smem,
                             cudaStream_t s) {
  const bool q8 = dtype == MINQ_Q8_0;
  switch (p.tp_world) {
    case 1: return q8 ? mk_launch_inst<MINQ_Q8_0, 1>(p, grid, smem, s) : mk_launch_inst<MINQ_Q4_0, 1>(p, grid, smem, s);
    case 2: return q8 ? mk_launch_inst<MINQ_Q8_0, 2>(p, grid, smem, s) : mk_launch_inst<MINQ_Q4_0, 2>(p, grid, smem, s);
    case 4: return q8 ? mk_launch_inst<MINQ_Q8_0, 4>(p, grid, smem, s) : mk_launch_inst<MINQ_Q4_0, 4>(p, grid, smem, s);
    case 8: return q8 ? mk_launch_inst<MINQ_Q8_0, 8>(p, grid, smem, s) : mk_launch_inst<MINQ_Q4_0, 8>(p, grid, smem, s);
    default: return fail(MINQ_ERR_ARG, "decode megakernel: 1, 2, 4 or 8 tensor-parallel ranks");
  }
}

}  // namespace minq
