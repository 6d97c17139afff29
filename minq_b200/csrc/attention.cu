// Decode attention over the HBM-resident f32 KV cache (model.rs:223-248
// `attend`, with the RoPE / Qwen3 q-k RMSNorm / cache append of
// forward_token, model.rs:291-303, in a small pre-kernel).
//
// Split-KV flash-decode:
//   * grid = (splits, n_kv * ceil(G/8), batch): one CTA owns one KV head, up
//     to 8 of the G query heads that share it (GQA, model.rs:226,232), and a
//     chunk of positions. K and V are each read from HBM exactly once per
//     query-head group.
//   * QK^T: 8-element lane slices (HD/8 lanes per position), float4 loads of
//     K that are contiguous across the lanes of a position, a shuffle
//     reduction inside the position's lane group; the query slice for every
//     head of the group lives in registers.
//   * Online softmax per warp over tiles of 32 positions (lane t owns
//     position t of the tile), exp via expf, running max / sum rescaling.
//   * PV: lanes split head_dim (float4 for HD=128), V rows are read fully
//     coalesced, the probability of position t is broadcast by a shuffle.
//   * Warps of a CTA merge their (max, sum, out) in shared memory; CTAs of a
//     split write unnormalised partials to the workspace and a combine kernel
//     merges the splits. With one split the CTA writes the output directly.
#include <math.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "ktimer.h"
#include "pipeline.cuh"

namespace minq {

struct AttnParams {
  const float* q;        // [B, nh, HD] rotated queries
  const float* k;        // cache base
  const float* v;
  size_t seq_stride, head_stride, pos_stride;  // element strides of the cache
  int nh, nkv, len, chunk, nsplit;
  float scale;           // 1/sqrt(HD)
  float* out;            // [B, nh, HD]
  float* ws_o;           // [B, nh, nsplit, HD]
  float* ws_ml;          // [B, nh, ws_stride, 2]
  int* status;           // device status word (bounded-wait timeouts)
  const int* d_pos;      // if set: len = *d_pos + 1 and the split is derived on the device
  int ws_stride;         // split slots per (sequence, head) in the workspace
  int q_round;           // chunk granularity (positions)
  int len_step;          // entry b attends over len + b * len_step positions
};

// Split of `len` positions into at most `cap` chunks of a multiple of `q`.
__device__ __forceinline__ void derive_split(int len, int cap, int q, int* chunk, int* nsplit) {
  int c = (len + cap - 1) / cap;
  c = (c + q - 1) / q * q;
  *chunk = c;
  *nsplit = (len + c - 1) / c;
}

template <int HD, int GMAX>
__global__ void __launch_bounds__(128) attn_split_kernel(AttnParams p) {
  constexpr int EPL = 8;                       // elements per lane in QK
  constexpr int LPP = HD / EPL;                // lanes per position (1..32)
  constexpr int PPS = 32 / LPP;                // positions per sub-step
  constexpr int DPL = HD >= 32 ? HD / 32 : 1;  // PV dims per lane
  constexpr int PV_LANES = HD / DPL;           // lanes active in PV
  static_assert(HD % 8 == 0 && HD <= 256, "head_dim");

  __shared__ float s_sc[4][GMAX][32];
  __shared__ float s_m[4][GMAX], s_l[4][GMAX];
  __shared__ float s_o[4][GMAX][HD];

  pdl_wait();
  pdl_launch_dependents();
  int len = p.len + (int)blockIdx.z * p.len_step, chunk = p.chunk, nsplit = p.nsplit;
  if (p.d_pos) {
    len = *p.d_pos + 1;
    derive_split(len, gridDim.x, p.q_round, &chunk, &nsplit);
  }
  const int split = blockIdx.x;
  if (split >= nsplit) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int b = blockIdx.z;
  const int G = p.nh / p.nkv;
  const int qgroups = (G + 7) / 8;
  const int kvh = blockIdx.y / qgroups;
  const int g0 = (blockIdx.y % qgroups) * 8;
  const int ng = min(GMAX, G - g0);
  const int t_begin = split * chunk;
  const int t_end = max(t_begin, min(len, t_begin + chunk));  // empty past an entry's length

  const float* kb = p.k + b * p.seq_stride + kvh * p.head_stride;
  const float* vb = p.v + b * p.seq_stride + kvh * p.head_stride;

  // Query slices: lane part j owns elements [4j, 4j+4) and [HD/2 + 4j, ...)
  // for HD >= 16 (two float4 per lane), or all 8 elements for HD == 8.
  const int j = lane % LPP;
  const int pslot = lane / LPP;
  float qr[GMAX][EPL];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    const float* qh = p.q + ((size_t)b * p.nh + kvh * G + g0 + (g < ng ? g : 0)) * HD;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      int idx = HD >= 16 ? ((e < 4) ? 4 * j + e : HD / 2 + 4 * j + e - 4) : e;
      qr[g][e] = g < ng ? qh[idx] * p.scale : 0.0f;
    }
  }

  float m_w[GMAX], l_w[GMAX], o[GMAX][DPL];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m_w[g] = -INFINITY;
    l_w[g] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) o[g][d] = 0.0f;
  }

  for (int tile = t_begin + warp * 32; tile < t_end; tile += nwarps * 32) {
    // --- scores for the 32 positions of this tile ---
#pragma unroll 2
    for (int ss = 0; ss < 32 / PPS; ++ss) {
      const int tl = ss * PPS + pslot;  // tile-local position
      const int t = tile + tl;
      float kv[EPL];
      if (t < t_end) {
        const float* kt = kb + (size_t)t * p.pos_stride;
        if constexpr (HD >= 16) {
          float4 a = *reinterpret_cast<const float4*>(kt + 4 * j);
          float4 c = *reinterpret_cast<const float4*>(kt + HD / 2 + 4 * j);
          kv[0] = a.x; kv[1] = a.y; kv[2] = a.z; kv[3] = a.w;
          kv[4] = c.x; kv[5] = c.y; kv[6] = c.z; kv[7] = c.w;
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) kv[e] = kt[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) kv[e] = 0.0f;
      }
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) s = fmaf(qr[g][e], kv[e], s);
#pragma unroll
        for (int off = LPP / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (j == 0) s_sc[warp][g][tl] = t < t_end ? s : -INFINITY;
      }
    }
    __syncwarp();
    // --- online softmax over the tile; lane owns position `lane` ---
    float pr[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      const float s = s_sc[warp][g][lane];
      const float mt = warp_max(s);
      const float mn = fmaxf(m_w[g], mt);
      const float corr = m_w[g] == -INFINITY ? 0.0f : expf(m_w[g] - mn);
      pr[g] = s == -INFINITY ? 0.0f : expf(s - mn);
      l_w[g] = l_w[g] * corr + pr[g];
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[g][d] *= corr;
      m_w[g] = mn;
    }
    __syncwarp();
    // --- PV ---
    const int nt = min(32, t_end - tile);
    for (int tl = 0; tl < nt; ++tl) {
      const float* vt = vb + (size_t)(tile + tl) * p.pos_stride;
      float vv[DPL];
      if (lane < PV_LANES) {
        if constexpr (DPL == 4) {
          float4 a = *reinterpret_cast<const float4*>(vt + 4 * lane);
          vv[0] = a.x; vv[1] = a.y; vv[2] = a.z; vv[3] = a.w;
        } else if constexpr (DPL == 2) {
          float2 a = *reinterpret_cast<const float2*>(vt + 2 * lane);
          vv[0] = a.x; vv[1] = a.y;
        } else {
#pragma unroll
          for (int d = 0; d < DPL; ++d) vv[d] = vt[DPL * lane + d];
        }
      } else {
#pragma unroll
        for (int d = 0; d < DPL; ++d) vv[d] = 0.0f;
      }
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        const float pt = __shfl_sync(0xffffffffu, pr[g], tl);
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[g][d] = fmaf(pt, vv[d], o[g][d]);
      }
    }
  }

  // --- merge warps ---
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    const float lsum = warp_sum(l_w[g]);
    if (lane == 0) {
      s_m[warp][g] = m_w[g];
      s_l[warp][g] = lsum;
    }
    if (lane < PV_LANES) {
#pragma unroll
      for (int d = 0; d < DPL; ++d) s_o[warp][g][DPL * lane + d] = o[g][d];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < ng * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (int w = 0; w < nwarps; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.0f, O = 0.0f;
    for (int w = 0; w < nwarps; ++w) {
      if (s_m[w][g] == -INFINITY) continue;
      const float f = expf(s_m[w][g] - M);
      L = fmaf(s_l[w][g], f, L);
      O = fmaf(s_o[w][g][d], f, O);
    }
    const int qh = kvh * G + g0 + g;
    const size_t row = (size_t)b * p.nh + qh;
    if (nsplit == 1) {
      p.out[row * HD + d] = O / L;
    } else {
      p.ws_o[(row * p.ws_stride + split) * HD + d] = O;
      if (d == 0) {
        p.ws_ml[(row * p.ws_stride + split) * 2 + 0] = M;
        p.ws_ml[(row * p.ws_stride + split) * 2 + 1] = L;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA-fed variant for caches whose positions are contiguous per KV head
// (pos_stride == HD, the model's head-major layout). CTA = 4 consumer warps
// + 1 producer warp. The producer streams K and V tiles of TP positions
// (TP*HD*4 = 8 KB each) into an 8-deep shared-memory ring with one bulk copy
// per tile; consumer warp w takes tiles w, w+4, ... and runs the same QK^T /
// online-softmax / PV math as attn_split_kernel from shared memory.
template <int HD>
struct TmaAttnCfg {
  static constexpr int TP = (2048 / HD) < 32 ? (2048 / HD) : 32;  // positions per tile
  // ring depth: a multiple of the 4 consumer warps (warp w takes tiles w,
  // w + 4, ...), so each slot is only ever used by one warp and its parity
  // waits see consecutive phases; 4 slots keep two CTAs per SM resident
  static constexpr int S = 4;
  static constexpr int TILE_FLOATS = TP * HD;
};

// Per-lane layout of the TMA-fed kernels' consumer warps (see below).
template <int HD>
struct TmaLanes {
  static constexpr int EPL = 8;                       // q / K elements per lane in QK
  static constexpr int LPP = HD / EPL;                // lanes per position
  static constexpr int PPS = 32 / LPP;                // positions per sub-step
  static constexpr int NSUB = TmaAttnCfg<HD>::TP / PPS;
  static constexpr int DPL = HD >= 32 ? HD / 32 : 1;  // PV dims per lane
  static constexpr int PV_LANES = HD / DPL;
};

// This lane's slice of the (pre-scaled) queries of heads g0 .. g0+ng-1 of
// sequence b's kv head kvh.
template <int HD, int GMAX>
__device__ __forceinline__ void tma_load_q(const AttnParams& p, int b, int kvh, int G, int g0,
                                           int ng, int j, float (&qr)[GMAX][TmaLanes<HD>::EPL]) {
  using LN = TmaLanes<HD>;
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    const float* qh = p.q + ((size_t)b * p.nh + kvh * G + g0 + (g < ng ? g : 0)) * HD;
#pragma unroll
    for (int e = 0; e < LN::EPL; ++e) {
      const int idx = (e < 4) ? 4 * j + e : HD / 2 + 4 * j + e - 4;
      qr[g][e] = g < ng ? qh[idx] * p.scale : 0.0f;
    }
  }
}

// One tile of npos positions (K rows kt_s, V rows vt_s in shared memory):
// QK^T for every head of the group, the online-softmax update of this
// warp's running max / sum, and p V into the warp's outputs.
template <int HD, int GMAX>
__device__ __forceinline__ void tma_attn_tile(const float (&qr)[GMAX][TmaLanes<HD>::EPL],
                                              const float* kt_s, const float* vt_s, int npos,
                                              float* sc, float (&m_w)[GMAX], float (&l_w)[GMAX],
                                              float (&o)[GMAX][TmaLanes<HD>::DPL]) {
  using LN = TmaLanes<HD>;
  constexpr int TP = TmaAttnCfg<HD>::TP, EPL = LN::EPL, LPP = LN::LPP, PPS = LN::PPS,
                NSUB = LN::NSUB, DPL = LN::DPL, PV_LANES = LN::PV_LANES;
  const int lane = threadIdx.x & 31, j = lane % LPP, pslot = lane / LPP;
#pragma unroll 2
  for (int ss = 0; ss < NSUB; ++ss) {
    const int tl = ss * PPS + pslot;
    const float* kt = kt_s + tl * HD;
    const float4 a = *reinterpret_cast<const float4*>(kt + 4 * j);
    const float4 c = *reinterpret_cast<const float4*>(kt + HD / 2 + 4 * j);
    const float kv[EPL] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      float sv = 0.0f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) sv = fmaf(qr[g][e], kv[e], sv);
#pragma unroll
      for (int off = LPP / 2; off > 0; off >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, off);
      if (j == 0) sc[g * 32 + tl] = tl < npos ? sv : -INFINITY;
    }
  }
  __syncwarp();
  float pr[GMAX];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    const float sv = lane < TP ? sc[g * 32 + lane] : -INFINITY;
    const float mt = warp_max(sv);
    const float mn = fmaxf(m_w[g], mt);
    const float corr = m_w[g] == -INFINITY ? 0.0f : expf(m_w[g] - mn);
    pr[g] = sv == -INFINITY ? 0.0f : expf(sv - mn);
    l_w[g] = l_w[g] * corr + pr[g];
#pragma unroll
    for (int d = 0; d < DPL; ++d) o[g][d] *= corr;
    m_w[g] = mn;
  }
#pragma unroll 4
  for (int tl = 0; tl < npos; ++tl) {
    const float* vt = vt_s + tl * HD;
    float vv[DPL];
    if (lane < PV_LANES) {
      if constexpr (DPL == 4) {
        const float4 a = *reinterpret_cast<const float4*>(vt + 4 * lane);
        vv[0] = a.x; vv[1] = a.y; vv[2] = a.z; vv[3] = a.w;
      } else if constexpr (DPL == 2) {
        const float2 a = *reinterpret_cast<const float2*>(vt + 2 * lane);
        vv[0] = a.x; vv[1] = a.y;
      } else {
#pragma unroll
        for (int d = 0; d < DPL; ++d) vv[d] = vt[DPL * lane + d];
      }
    } else {
#pragma unroll
      for (int d = 0; d < DPL; ++d) vv[d] = 0.0f;
    }
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      const float pt = __shfl_sync(0xffffffffu, pr[g], tl);
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[g][d] = fmaf(pt, vv[d], o[g][d]);
    }
  }
  __syncwarp();
}

// A warp's running (max, sum, out) per head into shared memory for the
// CTA's merge (s_m / s_l: [warp][GMAX], s_o: [warp][GMAX][HD]).
template <int HD, int GMAX>
__device__ __forceinline__ void tma_store_warp_state(int warp, const float (&m_w)[GMAX],
                                                     const float (&l_w)[GMAX],
                                                     const float (&o)[GMAX][TmaLanes<HD>::DPL],
                                                     float* s_m, float* s_l, float* s_o) {
  using LN = TmaLanes<HD>;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    const float lsum = warp_sum(l_w[g]);
    if (lane == 0) {
      s_m[warp * GMAX + g] = m_w[g];
      s_l[warp * GMAX + g] = lsum;
    }
    if (lane < LN::PV_LANES) {
#pragma unroll
      for (int d = 0; d < LN::DPL; ++d) s_o[(warp * GMAX + g) * HD + LN::DPL * lane + d] = o[g][d];
    }
  }
}

// Merge of the 4 consumer warps' states for output element idx = g * HD + d:
// the unnormalised sum O, its max M and sum L.
template <int HD, int GMAX>
__device__ __forceinline__ void tma_merge_warps(int idx, const float* s_m, const float* s_l,
                                                const float* s_o, float* O_, float* M_, float* L_) {
  const int g = idx / HD, d = idx % HD;
  float M = -INFINITY;
  for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w * GMAX + g]);
  float L = 0.0f, O = 0.0f;
  for (int w = 0; w < 4; ++w) {
    const float mw = s_m[w * GMAX + g];
    if (mw == -INFINITY) continue;
    const float f = expf(mw - M);
    L = fmaf(s_l[w * GMAX + g], f, L);
    O = fmaf(s_o[(w * GMAX + g) * HD + d], f, O);
  }
  *O_ = O;
  *M_ = M;
  *L_ = L;
}

template <int HD, int GMAX>
__global__ void __launch_bounds__(160) attn_tma_kernel(AttnParams p) {
  using CFG = TmaAttnCfg<HD>;
  constexpr int TP = CFG::TP, S = CFG::S, TF = CFG::TILE_FLOATS;
  constexpr int NWC = 4;                       // consumer warps
  static_assert(S % NWC == 0, "every ring slot must belong to one consumer warp");
  constexpr int EPL = TmaLanes<HD>::EPL, LPP = TmaLanes<HD>::LPP, DPL = TmaLanes<HD>::DPL;
  static_assert(HD >= 16 && HD <= 256 && TP % TmaLanes<HD>::PPS == 0, "head_dim");

  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + S;
  float* tiles = reinterpret_cast<float*>(smem_raw + 128);            // [S][2][TF]
  float* s_sc = tiles + (size_t)S * 2 * TF;                            // [NWC][GMAX][32]
  float* s_m = s_sc + NWC * GMAX * 32;                                 // [NWC][GMAX]
  float* s_l = s_m + NWC * GMAX;                                       // [NWC][GMAX]
  float* s_o = s_l + NWC * GMAX;                                       // [NWC][GMAX][HD]

  pdl_wait();  // K/V (this position) and q come from the previous kernel
  pdl_launch_dependents();
  int len = p.len + (int)blockIdx.z * p.len_step, chunk = p.chunk, nsplit = p.nsplit;
  if (p.d_pos) {
    len = *p.d_pos + 1;
    derive_split(len, gridDim.x, p.q_round, &chunk, &nsplit);
  }
  const int split = blockIdx.x;
  if (split >= nsplit) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.z;
  const int G = p.nh / p.nkv;
  const int qgroups = (G + 7) / 8;
  const int kvh = blockIdx.y / qgroups;
  const int g0 = (blockIdx.y % qgroups) * 8;
  const int ng = min(GMAX, G - g0);
  const int t_begin = split * chunk;
  const int t_end = max(t_begin, min(len, t_begin + chunk));  // empty past an entry's length
  const int ntiles = (t_end - t_begin + TP - 1) / TP;
  const float* kb = p.k + b * p.seq_stride + kvh * p.head_stride;
  const float* vb = p.v + b * p.seq_stride + kvh * p.head_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == NWC) {  // producer
    bool ok = true;
    for (int i = 0; i < ntiles && ok; ++i) {
      const int s = i % S;
      ok = mbar_wait(&empty[s], ((uint32_t)(i / S) & 1u) ^ 1u, p.status);
      if (!ok) break;
      const int t0 = t_begin + i * TP;
      const uint32_t bytes = (uint32_t)(min(TP, t_end - t0) * HD * 4);
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], 2 * bytes);
        bulk_g2s(tiles + (size_t)s * 2 * TF, kb + (size_t)t0 * HD, bytes, &full[s]);
        bulk_g2s(tiles + (size_t)s * 2 * TF + TF, vb + (size_t)t0 * HD, bytes, &full[s]);
      }
      __syncwarp();
    }
    for (int i = max(0, ntiles - S); ok && i < ntiles; ++i)
      ok = mbar_wait(&empty[i % S], (uint32_t)(i / S) & 1u, p.status);
  } else {
    float qr[GMAX][EPL];
    tma_load_q<HD, GMAX>(p, b, kvh, G, g0, ng, lane % LPP, qr);
    float m_w[GMAX], l_w[GMAX], o[GMAX][DPL];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      m_w[g] = -INFINITY;
      l_w[g] = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[g][d] = 0.0f;
    }
    float* sc = s_sc + warp * GMAX * 32;
    for (int i = warp; i < ntiles; i += NWC) {
      const int s = i % S;
      if (!mbar_wait(&full[s], (uint32_t)(i / S) & 1u, p.status)) break;
      const float* kt_s = tiles + (size_t)s * 2 * TF;
      const int npos = min(TP, t_end - (t_begin + i * TP));
      tma_attn_tile<HD, GMAX>(qr, kt_s, kt_s + TF, npos, sc, m_w, l_w, o);
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    tma_store_warp_state<HD, GMAX>(warp, m_w, l_w, o, s_m, s_l, s_o);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < ng * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float O, M, L;
    tma_merge_warps<HD, GMAX>(idx, s_m, s_l, s_o, &O, &M, &L);
    const size_t row = (size_t)b * p.nh + kvh * G + g0 + g;
    if (nsplit == 1) {
      p.out[row * HD + d] = O / L;
    } else {
      p.ws_o[(row * p.ws_stride + split) * HD + d] = O;
      if (d == 0) {
        p.ws_ml[(row * p.ws_stride + split) * 2 + 0] = M;
        p.ws_ml[(row * p.ws_stride + split) * 2 + 1] = L;
      }
    }
  }
}

template <int HD, int GMAX>
static size_t tma_attn_smem() {
  using CFG = TmaAttnCfg<HD>;
  return 128 + sizeof(float) * ((size_t)CFG::S * 2 * CFG::TILE_FLOATS + 4 * GMAX * 32 +
                                2 * 4 * GMAX + 4 * GMAX * HD);
}

// ---------------------------------------------------------------------------
// Balanced ("stream-K") form of the TMA-fed kernel for histories of one
// host-known length. The work is the list of T = units x NT tiles, unit u =
// (sequence, kv head, query group) with NT tiles of TP positions each, in
// that order; CTA c of the G CTAs (a fixed number per SM) takes tiles
// [c T / G, (c + 1) T / G), so every SM streams the same number of bytes and
// the grid ends in one wave, whatever the batch and length. A CTA's range
// may cross units: at each unit boundary its warps merge their states and
// write the unit's partial into slot c - c_first(u) of the unit's rows
// (c_first(u): the CTA holding the unit's first tile); the combine kernel
// merges a unit's slots c_first(u) .. c_last(u). The ring protocol and the
// tile arithmetic are those of attn_tma_kernel (consumer warp w takes the
// range's tiles w, w + 4, ...).
struct SkPlan {
  long long T;  // tiles in all
  int NT;       // tiles per unit
  int G;        // CTAs
};

// The CTA whose range holds tile t: the largest c with floor(c T / G) <= t.
__device__ __host__ __forceinline__ int sk_cta_of(long long t, const SkPlan& k) {
  return (int)(((t + 1) * k.G - 1) / k.T);
}

template <int HD, int GMAX>
__global__ void __launch_bounds__(160) attn_sk_kernel(AttnParams p, SkPlan k) {
  using CFG = TmaAttnCfg<HD>;
  constexpr int TP = CFG::TP, S = CFG::S, TF = CFG::TILE_FLOATS;
  constexpr int NWC = 4;
  static_assert(S % NWC == 0, "every ring slot must belong to one consumer warp");
  constexpr int EPL = TmaLanes<HD>::EPL, LPP = TmaLanes<HD>::LPP, DPL = TmaLanes<HD>::DPL;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + S;
  float* tiles = reinterpret_cast<float*>(smem_raw + 128);  // [S][2][TF]
  float* s_sc = tiles + (size_t)S * 2 * TF;                  // [NWC][GMAX][32]
  float* s_m = s_sc + NWC * GMAX * 32;                       // [NWC][GMAX]
  float* s_l = s_m + NWC * GMAX;                             // [NWC][GMAX]
  float* s_o = s_l + NWC * GMAX;                             // [NWC][GMAX][HD]

  pdl_wait();  // K/V (this position) and q come from the previous kernel
  pdl_launch_dependents();
  const long long r0 = (long long)blockIdx.x * k.T / k.G;
  const long long r1 = (long long)(blockIdx.x + 1) * k.T / k.G;
  if (r1 <= r0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.nh / p.nkv, qgroups = (G + 7) / 8, len = p.len;
  // unit u -> (sequence, kv head, first query head of the group)
  auto unit = [&](long long u, int* b, int* kvh, int* g0) {
    *g0 = (int)(u % qgroups) * 8;
    *kvh = (int)((u / qgroups) % p.nkv);
    *b = (int)(u / ((long long)qgroups * p.nkv));
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  const int n = (int)(r1 - r0);  // tiles of this CTA
  if (warp == NWC) {  // producer: the range's tiles in order, across units
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int s = i % S;
      ok = mbar_wait(&empty[s], ((uint32_t)(i / S) & 1u) ^ 1u, p.status);
      if (!ok) break;
      const long long t = r0 + i;
      int b, kvh, g0;
      unit(t / k.NT, &b, &kvh, &g0);
      const int pos0 = (int)(t % k.NT) * TP;
      const uint32_t bytes = (uint32_t)(min(TP, len - pos0) * HD * 4);
      if (lane == 0) {
        const size_t off = (size_t)b * p.seq_stride + (size_t)kvh * p.head_stride + (size_t)pos0 * HD;
        mbar_arrive_expect_tx(&full[s], 2 * bytes);
        bulk_g2s(tiles + (size_t)s * 2 * TF, p.k + off, bytes, &full[s]);
        bulk_g2s(tiles + (size_t)s * 2 * TF + TF, p.v + off, bytes, &full[s]);
      }
      __syncwarp();
    }
    for (int i = max(0, n - S); ok && i < n; ++i)
      ok = mbar_wait(&empty[i % S], (uint32_t)(i / S) & 1u, p.status);
    return;
  }
  // consumers: one segment (the range's part of one unit) at a time
  bool ok = true;
  float* sc = s_sc + warp * GMAX * 32;
  for (long long u = r0 / k.NT; u * k.NT < r1; ++u) {
    const long long a = max(r0, u * k.NT), e = min(r1, (u + 1) * k.NT);
    int b, kvh, g0;
    unit(u, &b, &kvh, &g0);
    const int ng = min(GMAX, G - g0);
    float qr[GMAX][EPL];
    tma_load_q<HD, GMAX>(p, b, kvh, G, g0, ng, lane % LPP, qr);
    float m_w[GMAX], l_w[GMAX], o[GMAX][DPL];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      m_w[g] = -INFINITY;
      l_w[g] = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[g][d] = 0.0f;
    }
    // this warp's tiles of the segment: range indices i = t - r0 with i = warp mod 4
    const int ia = (int)(a - r0), ie = (int)(e - r0);
    for (int i = ia + ((warp - ia % NWC) + NWC) % NWC; ok && i < ie; i += NWC) {
      const int s = i % S;
      if (!(ok = mbar_wait(&full[s], (uint32_t)(i / S) & 1u, p.status))) break;
      const float* kt_s = tiles + (size_t)s * 2 * TF;
      const int pos0 = (int)((r0 + i) % k.NT) * TP;
      tma_attn_tile<HD, GMAX>(qr, kt_s, kt_s + TF, min(TP, len - pos0), sc, m_w, l_w, o);
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    tma_store_warp_state<HD, GMAX>(warp, m_w, l_w, o, s_m, s_l, s_o);
    named_barrier_sync(1, 32 * NWC);
    const int slot = (int)blockIdx.x - sk_cta_of(u * k.NT, k);
    for (int idx = threadIdx.x; idx < ng * HD; idx += 32 * NWC) {
      const int g = idx / HD, d = idx % HD;
      float O, M, L;
      tma_merge_warps<HD, GMAX>(idx, s_m, s_l, s_o, &O, &M, &L);
      const size_t row = (size_t)b * p.nh + kvh * G + g0 + g;
      p.ws_o[(row * p.ws_stride + slot) * HD + d] = O;
      if (d == 0) {
        p.ws_ml[(row * p.ws_stride + slot) * 2 + 0] = M;
        p.ws_ml[(row * p.ws_stride + slot) * 2 + 1] = L;
      }
    }
    named_barrier_sync(1, 32 * NWC);  // the warp states are rewritten by the next segment
  }
}

// Merge of every (sequence, query head)'s stream-K slots: the CTAs that
// covered its unit, c_first .. c_last.
__global__ void attn_sk_combine_kernel(const float* ws_o, const float* ws_ml, SkPlan k, int nh,
                                       int nkv, int stride, int hd, float* out) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t row = blockIdx.x;  // b * nh + h
  const int G = nh / nkv, qgroups = (G + 7) / 8;
  const int b = (int)(row / nh), h = (int)(row % nh);
  const long long u = ((long long)b * nkv + h / G) * qgroups + (h % G) / 8;
  const int nslot = sk_cta_of(u * k.NT + k.NT - 1, k) - sk_cta_of(u * k.NT, k) + 1;
  const float* ml = ws_ml + row * stride * 2;
  float M = -INFINITY;
  for (int s = 0; s < nslot; ++s) M = fmaxf(M, ml[2 * s]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < nslot; ++s) {
      const float m = ml[2 * s];
      if (m == -INFINITY) continue;
      const float f = expf(m - M);
      L = fmaf(ml[2 * s + 1], f, L);
      O = fmaf(ws_o[(row * stride + s) * hd + d], f, O);
    }
    out[row * hd + d] = O / L;
  }
}

// Merge the splits of every (sequence, query head).
__global__ void attn_combine_kernel(const float* ws_o, const float* ws_ml, int nsplit, int stride,
                                    int hd, float* out, const int* d_pos, int cap, int q) {
  pdl_wait();
  pdl_launch_dependents();
  if (d_pos) {
    int chunk;
    derive_split(*d_pos + 1, cap, q, &chunk, &nsplit);
    if (nsplit == 1) return;  // the split kernel wrote the output directly
  }
  const size_t row = blockIdx.x;  // b * nh + h
  const float* ml = ws_ml + row * stride * 2;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ml[2 * s]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
      const float m = ml[2 * s];
      if (m == -INFINITY) continue;
      const float f = expf(m - M);
      L = fmaf(ml[2 * s + 1], f, L);
      O = fmaf(ws_o[(row * stride + s) * hd + d], f, O);
    }
    out[row * hd + d] = O / L;
  }
}

// Per-head RMSNorm (model.rs:206-216), RoPE from tables (model.rs:189-201),
// and the cache append (model.rs:300-301). grid = (nh + 2*nkv heads, B);
// one warp per head.
struct RopeParams {
  const float* q_in;   // [B, nh, HD]
  const float* k_in;   // [B, nkv, HD]
  const float* v_in;   // [B, nkv, HD]
  size_t q_in_bstride, kv_in_bstride;  // element stride between sequences
  const float* q_norm;
  const float* k_norm;
  float eps;
  const float* cos_t;  // [max_seq, HD/2]
  const float* sin_t;
  int nh, nkv, hd, pos;
  int pos_step;        // entry b takes position pos + b * pos_step
  const int* d_pos;    // if set, the position is read from the device
  float* q_out;        // [B, nh, HD]
  float* k_cache;
  float* v_cache;
  size_t seq_stride, head_stride, pos_stride;
};

__global__ void rope_append_kernel(RopeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int pos = (p.d_pos ? *p.d_pos : p.pos) + b * p.pos_step;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nheads = p.nh + 2 * p.nkv;
  if (head >= nheads) return;
  const int hd = p.hd, half = hd / 2;
  float vals[8];  // hd <= 256
  const float* src;
  const float* gain = nullptr;
  float* dst;
  bool rope = true;
  if (head < p.nh) {
    src = p.q_in + b * p.q_in_bstride + (size_t)head * hd;
    gain = p.q_norm;
    dst = p.q_out + ((size_t)b * p.nh + head) * hd;
  } else if (head < p.nh + p.nkv) {
    const int h = head - p.nh;
    src = p.k_in + b * p.kv_in_bstride + (size_t)h * hd;
    gain = p.k_norm;
    dst = p.k_cache + b * p.seq_stride + h * p.head_stride + (size_t)pos * p.pos_stride;
  } else {
    const int h = head - p.nh - p.nkv;
    src = p.v_in + b * p.kv_in_bstride + (size_t)h * hd;
    dst = p.v_cache + b * p.seq_stride + h * p.head_stride + (size_t)pos * p.pos_stride;
    rope = false;
  }
  // Lane owns element pairs (i, i + half) for i = lane, lane + 32, ...
  const int npairs = (half + 31) / 32;
  for (int k = 0; k < npairs; ++k) {
    const int i = lane + 32 * k;
    vals[2 * k] = i < half ? src[i] : 0.0f;
    vals[2 * k + 1] = i < half ? src[i + half] : 0.0f;
  }
  if (gain) {
    float ss = 0.0f;
    for (int k = 0; k < npairs; ++k) ss = fmaf(vals[2 * k], vals[2 * k], fmaf(vals[2 * k + 1], vals[2 * k + 1], ss));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + p.eps);
    for (int k = 0; k < npairs; ++k) {
      const int i = lane + 32 * k;
      if (i < half) {
        vals[2 * k] = vals[2 * k] * inv * gain[i];
        vals[2 * k + 1] = vals[2 * k + 1] * inv * gain[i + half];
      }
    }
  }
  for (int k = 0; k < npairs; ++k) {
    const int i = lane + 32 * k;
    if (i >= half) continue;
    float x1 = vals[2 * k], x2 = vals[2 * k + 1];
    if (rope) {
      const float c = p.cos_t[(size_t)pos * half + i];
      const float s = p.sin_t[(size_t)pos * half + i];
      // head[i] = x1*cos - x2*sin; head[i+half] = x2*cos + x1*sin (un-fused)
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      x1 = y1;
      x2 = y2;
    }
    dst[i] = x1;
    dst[i + half] = x2;
  }
}

// ---------------------------------------------------------------------------

static int pick_chunk(int len, size_t units) {
  const size_t target = (size_t)sm_count() * 8;
  size_t c = ((size_t)len * units + target - 1) / target;
  c = (c + 31) / 32 * 32;
  if (c < 32) c = 32;
  if (c > 4096) c = 4096;
  return (int)c;
}

// Split plan of launch_attention: positions per split (chunk) and the
// chunk granularity, for `batch` entries whose longest history is size_len.
static void attn_split_plan(bool tma, size_t batch, int nh, int nkv, int hd, int size_len,
                            int* chunk, int* q_round) {
  const int qgroups = (nh / nkv + 7) / 8;
  const size_t units = batch * nkv * qgroups;
  if (tma) {
    const int tp = std::min(32, 2048 / hd);
    *q_round = 4 * tp;
    const size_t target = (size_t)sm_count() * 2;
    size_t c = ((size_t)size_len * units + target - 1) / target;
    c = (c + *q_round - 1) / *q_round * *q_round;
    *chunk = (int)std::min<size_t>(c, (size_t)((size_len + *q_round - 1) / *q_round * *q_round));
  } else {
    *q_round = 32;
    *chunk = pick_chunk(size_len, units);
  }
}

size_t attn_workspace_need(size_t batch, int nh, int nkv, int hd, int size_len, bool head_major) {
  const bool tma = head_major && hd >= 16 && hd <= 256 && (hd & (hd - 1)) == 0;
  int chunk = 0, q_round = 0;
  attn_split_plan(tma, batch, nh, nkv, hd, size_len, &chunk, &q_round);
  const size_t nsplit = ((size_t)size_len + chunk - 1) / chunk;
  return nsplit > 1 ? batch * nh * nsplit * (hd + 2) * sizeof(float) : 0;
}

size_t attn_workspace_bytes(size_t batch, size_t nh, size_t len, size_t hd_max) {
  // Upper bound over every split choice: at most ceil(len / 32) splits.
  const size_t splits = (len + 31) / 32;
  return batch * nh * splits * (hd_max + 2) * sizeof(float) + 256;
}

template <int HD>
static minq_status launch_split_hd(const AttnParams& p, int gmax, dim3 grid, int threads,
                                   cudaStream_t s) {
  switch (gmax) {
    case 1: MINQ_CUDA_TRY(launch_k(attn_split_kernel<HD, 1>, grid, dim3(threads), 0, s, p)); break;
    case 2: MINQ_CUDA_TRY(launch_k(attn_split_kernel<HD, 2>, grid, dim3(threads), 0, s, p)); break;
    case 4: MINQ_CUDA_TRY(launch_k(attn_split_kernel<HD, 4>, grid, dim3(threads), 0, s, p)); break;
    default: MINQ_CUDA_TRY(launch_k(attn_split_kernel<HD, 8>, grid, dim3(threads), 0, s, p)); break;
  }
  return MINQ_OK;
}

template <int HD, int GMAX>
static minq_status launch_tma_inst(const AttnParams& p, dim3 grid, cudaStream_t s) {
  const size_t smem = tma_attn_smem<HD, GMAX>();
  auto k = attn_tma_kernel<HD, GMAX>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
  MINQ_CUDA_TRY(launch_k(k, grid, dim3(160), smem, s, p));
  return MINQ_OK;
}

template <int HD>
static minq_status launch_tma_hd(const AttnParams& p, int gmax, dim3 grid, cudaStream_t s) {
  switch (gmax) {
    case 1: return launch_tma_inst<HD, 1>(p, grid, s);
    case 2: return launch_tma_inst<HD, 2>(p, grid, s);
    case 4: return launch_tma_inst<HD, 4>(p, grid, s);
    default: return launch_tma_inst<HD, 8>(p, grid, s);
  }
}

template <int HD, int GMAX>
static minq_status launch_sk_inst(const AttnParams& p, const SkPlan& k, cudaStream_t s) {
  const size_t smem = tma_attn_smem<HD, GMAX>();
  auto kern = attn_sk_kernel<HD, GMAX>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  MINQ_CUDA_TRY(launch_k(kern, dim3((unsigned)k.G), dim3(160), smem, s, p, k));
  return MINQ_OK;
}

template <int HD>
static minq_status launch_sk_hd(const AttnParams& p, const SkPlan& k, int gmax, cudaStream_t s) {
  switch (gmax) {
    case 1: return launch_sk_inst<HD, 1>(p, k, s);
    case 2: return launch_sk_inst<HD, 2>(p, k, s);
    case 4: return launch_sk_inst<HD, 4>(p, k, s);
    default: return launch_sk_inst<HD, 8>(p, k, s);
  }
}

// The stream-K plan (attn_sk_kernel) for `batch` entries of `len` positions:
// three CTAs per SM (MINQ_ATTN_SK_CTAS: 1..3 per SM, 0 keeps the
// split-per-unit plan), taken when there are at least 16 units and 24
// tiles per CTA. Measured on B200 (GQA 32/8, head_dim 128), against the
// split-per-unit plan: B 64 / L 8192 4.42 -> 5.91 TB/s, B 64 / L 2048 3.97
// -> 5.15, B 8 / L 32768 4.67 -> 5.69, B 8 / L 8192 4.01 -> 4.51, B 64 /
// L 512 3.00 -> 3.50; slower below those sizes (one sequence: 2-35 %, its
// split plan already fills the SMs evenly; B 8 / L <= 2048: 4-20 %), and
// two CTAs per SM slower everywhere. False when the plan is not taken or
// the partial slots do not fit `ws_bytes`.
constexpr int kSkMinUnits = 16;
constexpr int kSkMinTilesPerCta = 24;
static bool attn_sk_plan(size_t batch, int nh, int nkv, int hd, int len, size_t ws_bytes,
                         SkPlan* k, int* stride) {
  static const int per_sm = [] {
    const char* e = std::getenv("MINQ_ATTN_SK_CTAS");
    return e ? std::max(0, std::min(3, std::atoi(e))) : 3;
  }();
  if (per_sm == 0 || len <= 0) return false;
  const int tp = std::min(32, 2048 / hd);
  const long long units = (long long)batch * nkv * ((nh / nkv + 7) / 8);
  k->NT = (len + tp - 1) / tp;
  k->T = units * k->NT;
  k->G = per_sm * sm_count();
  if (units < kSkMinUnits || k->T < (long long)kSkMinTilesPerCta * k->G) return false;
  int mx = 0;
  for (long long u = 0; u < units; ++u)
    mx = std::max(mx, sk_cta_of(u * k->NT + k->NT - 1, *k) - sk_cta_of(u * k->NT, *k) + 1);
  *stride = mx;
  return batch * nh * (size_t)mx * (hd + 2) * sizeof(float) <= ws_bytes;
}

// Decode attention over `len` positions (host-known), or, when `d_pos` is
// set, over *d_pos + 1 positions read on the device, with the grid sized
// for `cap_len` positions (a graph-captured step replays for any length up
// to the cache capacity).
minq_status launch_attention(const float* q, const float* k, const float* v, size_t batch,
                             int nh, int nkv, int hd, int len, size_t seq_stride,
                             size_t head_stride, size_t pos_stride, float* out, void* ws,
                             size_t ws_bytes, cudaStream_t s, const int* d_pos, int cap_len,
                             bool record_status, int len_step, int* status_word) {
  if (!d_pos && len <= 0) return fail(MINQ_ERR_SHAPE, "attention over an empty history");
  if (len_step < 0 || (len_step && d_pos))
    return fail(MINQ_ERR_ARG, "per-entry history lengths take host positions");
  if (nkv <= 0 || nh % nkv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  const int G = nh / nkv;
  const int qgroups = (G + 7) / 8;
  const int gmax = G > 4 ? 8 : (G > 2 ? 4 : (G > 1 ? 2 : 1));
  // sizes the grid: the longest entry
  const int size_len = (d_pos ? cap_len : len) + (int)(batch - 1) * len_step;
  AttnParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.seq_stride = seq_stride;
  p.head_stride = head_stride;
  p.pos_stride = pos_stride;
  p.nh = nh;
  p.nkv = nkv;
  p.len = len;
  p.len_step = len_step;
  p.status = !record_status ? nullptr : (status_word ? status_word : device_status_word());
  p.d_pos = d_pos;
  // The TMA path needs each KV head's positions contiguous (head-major
  // cache) and 16-byte aligned tiles.
  const bool tma = hd >= 16 && hd <= 256 && (hd & (hd - 1)) == 0 && pos_stride == (size_t)hd &&
                   (uintptr_t)k % 16 == 0 && (uintptr_t)v % 16 == 0 &&
                   seq_stride % 4 == 0 && head_stride % 4 == 0;
  // host-known histories of one length: the balanced stream-K plan
  SkPlan sk{};
  int sk_stride = 0;
  if (tma && !d_pos && len_step == 0 && ws &&
      attn_sk_plan(batch, nh, nkv, hd, len, ws_bytes, &sk, &sk_stride)) {
    p.scale = 1.0f / sqrtf((float)hd);
    p.out = out;
    p.ws_stride = sk_stride;
    p.ws_o = static_cast<float*>(ws);
    p.ws_ml = p.ws_o + batch * nh * (size_t)sk_stride * hd;
    ScopedKTimer timer(KF_ATTENTION, s, 8.0 * batch * nkv * hd * (double)len + 8.0 * batch * nh * hd);
    switch (hd) {
      case 16: MINQ_TRY(launch_sk_hd<16>(p, sk, gmax, s)); break;
      case 32: MINQ_TRY(launch_sk_hd<32>(p, sk, gmax, s)); break;
      case 64: MINQ_TRY(launch_sk_hd<64>(p, sk, gmax, s)); break;
      case 128: MINQ_TRY(launch_sk_hd<128>(p, sk, gmax, s)); break;
      default: MINQ_TRY(launch_sk_hd<256>(p, sk, gmax, s)); break;
    }
    MINQ_LAUNCH_CHECK("attn_sk_kernel");
    MINQ_CUDA_TRY(launch_k(attn_sk_combine_kernel, dim3((unsigned)(batch * nh)),
                           dim3(std::min(hd, 128)), 0, s, (const float*)p.ws_o,
                           (const float*)p.ws_ml, sk, nh, nkv, sk_stride, hd, out));
    MINQ_LAUNCH_CHECK("attn_sk_combine_kernel");
    return MINQ_OK;
  }
  attn_split_plan(tma, batch, nh, nkv, hd, size_len, &p.chunk, &p.q_round);
  p.nsplit = (size_len + p.chunk - 1) / p.chunk;  // grid (split slots)
  p.ws_stride = p.nsplit;
  p.scale = 1.0f / sqrtf((float)hd);
  p.out = out;
  const bool may_split = p.nsplit > 1;
  if (may_split) {
    const size_t need = batch * nh * p.nsplit * (hd + 2) * sizeof(float);
    if (!ws || ws_bytes < need)
      return fail(MINQ_ERR_ARG, "attention workspace too small (need " + std::to_string(need) +
                                    " bytes)");
    p.ws_o = static_cast<float*>(ws);
    p.ws_ml = p.ws_o + batch * nh * p.nsplit * hd;
  }
  const int threads = 32 * std::min(4, (p.chunk + 31) / 32);
  dim3 grid(p.nsplit, nkv * qgroups, (unsigned)batch);
  ScopedKTimer timer(KF_ATTENTION, s,
                     8.0 * batch * nkv * hd * (double)(d_pos ? cap_len : len) +
                         8.0 * batch * nh * hd);
  if (tma) {
    switch (hd) {
      case 16: MINQ_TRY(launch_tma_hd<16>(p, gmax, grid, s)); break;
      case 32: MINQ_TRY(launch_tma_hd<32>(p, gmax, grid, s)); break;
      case 64: MINQ_TRY(launch_tma_hd<64>(p, gmax, grid, s)); break;
      case 128: MINQ_TRY(launch_tma_hd<128>(p, gmax, grid, s)); break;
      default: MINQ_TRY(launch_tma_hd<256>(p, gmax, grid, s)); break;
    }
  } else {
    switch (hd) {
      case 8: MINQ_TRY(launch_split_hd<8>(p, gmax, grid, threads, s)); break;
      case 16: MINQ_TRY(launch_split_hd<16>(p, gmax, grid, threads, s)); break;
      case 32: MINQ_TRY(launch_split_hd<32>(p, gmax, grid, threads, s)); break;
      case 64: MINQ_TRY(launch_split_hd<64>(p, gmax, grid, threads, s)); break;
      case 128: MINQ_TRY(launch_split_hd<128>(p, gmax, grid, threads, s)); break;
      case 256: MINQ_TRY(launch_split_hd<256>(p, gmax, grid, threads, s)); break;
      default:
        return fail(MINQ_ERR_SHAPE, "unsupported head_dim " + std::to_string(hd) +
                                        " (supported: 8, 16, 32, 64, 128, 256)");
    }
  }
  MINQ_LAUNCH_CHECK("attn_split_kernel");
  if (may_split) {
    MINQ_CUDA_TRY(launch_k(attn_combine_kernel, dim3((unsigned)(batch * nh)),
                           dim3(std::min(hd, 128)), 0, s, (const float*)p.ws_o,
                           (const float*)p.ws_ml, p.nsplit, p.ws_stride, hd, out, d_pos,
                           (int)p.nsplit, p.q_round));
    MINQ_LAUNCH_CHECK("attn_combine_kernel");
  }
  return MINQ_OK;
}

minq_status launch_rope_append(const float* q_in, const float* k_in, const float* v_in,
                               size_t q_in_bstride, size_t kv_in_bstride, const float* q_norm,
                               const float* k_norm, float eps, const float* cos_t,
                               const float* sin_t, size_t batch, int nh, int nkv, int hd,
                               int pos, float* q_out, float* k_cache, float* v_cache,
                               size_t seq_stride, size_t head_stride, size_t pos_stride,
                               cudaStream_t s, const int* d_pos, int pos_step) {
  if (hd % 2 != 0 || hd > 256) return fail(MINQ_ERR_SHAPE, "head_dim must be even and <= 256");
  RopeParams p{};
  p.q_in = q_in;
  p.k_in = k_in;
  p.v_in = v_in;
  p.q_in_bstride = q_in_bstride;
  p.kv_in_bstride = kv_in_bstride;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.eps = eps;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.nh = nh;
  p.nkv = nkv;
  p.hd = hd;
  p.pos = pos;
  p.pos_step = pos_step;
  p.d_pos = d_pos;
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.seq_stride = seq_stride;
  p.head_stride = head_stride;
  p.pos_stride = pos_stride;
  const int heads = nh + 2 * nkv;
  dim3 grid((heads + 3) / 4, (unsigned)batch);
  MINQ_CUDA_TRY(launch_k(rope_append_kernel, grid, dim3(128), 0, s, p));
  MINQ_LAUNCH_CHECK("rope_append_kernel");
  return MINQ_OK;
}

}  // namespace minq
