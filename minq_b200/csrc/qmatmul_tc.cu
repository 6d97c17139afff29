// Tensor-core batched projections (the batched step from 2 inputs on):
// Y[b] = W X[b] for Q4_0 / Q8_0 weights with mma.sync m16n8k16 (bf16 in,
// f32 accumulate), the input RMSNorm (tensor.rs:219-227) applied first and
// bias / residual / SwiGLU after, the weights read once for all B inputs.
//
// Operands. Weight codes enter as exact bf16 values (Q4_0: nibble - 8, Q8_0:
// the i8 code). Each input is split into x_hi = bf16(x) and x_lo = bf16(x -
// x_hi) (16 significand bits together) and both parts run through the
// tensor cores, so a block's sum_k code_k x_k is exact up to the f32
// accumulation and the 2^-16 relative rounding of the split input. The
// block scale d is applied once per 32-column block with an f32 FMA into the
// row's running sum (quantize.rs:252-280: acc += d * sum).
//
// Layout. A 32-column block is two k-steps of 16; the k order inside a block
// is permuted so that lane (g, t) of a warp (g = lane / 4, t = lane mod 4)
// takes all of its A operand for both steps from one code word: columns
// 8t .. 8t + 7 (Q4_0: word t of the block's 16 code bytes; Q8_0: words 2t,
// 2t + 1). The inputs are written once per projection in the same permuted
// order (tc_xprep_kernel), so the B operand is a plain ldmatrix of rows of
// x_hi / x_lo.
//
// Work. A CTA of 8 warps takes 128 rows (64 rows of gate and of up for the
// dual form) and a slice of the columns; a warp owns 16 rows and every input
// (up to 8 n-tiles of 8). Chunks of 4 blocks of the CTA's rows and of the
// inputs' columns stream through a 4-deep ring in shared memory with
// cp.async (three chunks in flight while one is computed). With
// S > 1 column slices the partials go to the workspace and
// qmm_reduce-style summation in slice order applies the epilogue.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "matvec_common.cuh"
#include "pipeline.cuh"

namespace minq {

namespace {

constexpr int kTcWarps = 8;
constexpr int kTcThreads = 32 * kTcWarps;
constexpr int kTcBpc = 4;                 // blocks per chunk
constexpr int kTcKc = kTcBpc * kBlock;    // columns per chunk
constexpr int kTcMaxB = 64;
constexpr int kTcXPitch = kTcKc * 2 + 16;  // bytes per staged input row: ldmatrix rows on distinct banks
constexpr int kTcStages = 2;              // chunk buffers (kTcStages - 1 chunks in flight)
constexpr int kTcMinBlocks = 2;           // CTAs per SM (registers <= 128)

// Column of a 32-column block at k-step s (0, 1), k-slot kap (0..15) of the
// permuted order (see above).
__host__ __device__ constexpr int tc_col(int s, int kap) {
  return 8 * ((kap & 7) >> 1) + 4 * s + 2 * (kap >> 3) + (kap & 1);
}

struct TcParams {
  const uint8_t* w0;             // [rows][cols] blocks
  const uint8_t* w1;             // dual: up rows, else null
  size_t rows;
  int nb;                        // blocks per row (a multiple of kTcBpc)
  int B;
  const __nv_bfloat16* xh;       // [B][cols] permuted x_hi
  const __nv_bfloat16* xl;       // [B][cols] permuted x_lo
  int S;                         // column slices
  int slice_blocks;              // blocks per slice (a multiple of kTcBpc)
  const float* bias;             // [rows] or null
  const float* residual;         // [B][y_stride] or null (may alias y)
  float* y;                      // [B][y_stride]
  size_t y_stride;
  float* part;                   // S > 1: [S][halves][B][rows]
};

// x[b] -> permuted x_hi / x_lo (bf16), optionally RMSNorm'd first with the
// reference's f32 operations (x * inv * w). CTA (b, j) writes positions
// [1024 j, 1024 j + 1024) of input b, four per thread; with the norm every
// CTA of the input first sums the whole row's squares (float4 loads).
constexpr int kTcPrepCols = 1024;
__global__ void __launch_bounds__(256) tc_xprep_kernel(const float* __restrict__ x, size_t x_stride,
                                                      int n, const float* __restrict__ w, float eps,
                                                      __nv_bfloat16* __restrict__ xh,
                                                      __nv_bfloat16* __restrict__ xl) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[9];
  const float* row = x + (size_t)blockIdx.x * x_stride;
  float inv = 1.0f;
  if (w) {
    float ss = 0.0f;
    const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
    for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) {
      const float4 v = r4[i];
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = 0.0f;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) v += red[k];
      red[8] = 1.0f / sqrtf(v / (float)n + eps);
    }
    __syncthreads();
    inv = red[8];
  }
  __nv_bfloat16* oh = xh + (size_t)blockIdx.x * n;
  __nv_bfloat16* ol = xl + (size_t)blockIdx.x * n;
  const int p0 = blockIdx.y * kTcPrepCols;
  float v[4];
  int pp[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int p = p0 + threadIdx.x + 256 * k;
    pp[k] = p;
    v[k] = 0.0f;
    if (p < n) {
      const int q = p & 31;
      const int c = (p - q) + tc_col(q >> 4, q & 15);
      v[k] = w ? row[c] * inv * w[c] : row[c];
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (pp[k] >= n) continue;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v[k]);
    oh[pp[k]] = hi;
    ol[pp[k]] = __float2bfloat16_rn(v[k] - __bfloat162float(hi));
  }
}

__device__ __forceinline__ void tc_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void tc_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_stages() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kTcStages - 1) : "memory");
}
__device__ __forceinline__ void tc_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t tc_lds(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ void tc_ldsm4(uint32_t a, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void tc_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t tc_bits(__nv_bfloat162 v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}
__device__ __forceinline__ __nv_bfloat162 tc_bf2(uint32_t u) {
  __nv_bfloat162 v;
  memcpy(&v, &u, 4);
  return v;
}

// The two Q4_0 codes of byte e of word w (low nibble: the even column) as
// exact bf16 (code - 8): 0x4300 | c is bf16(128 + c), minus 136 (0x4308).
// w4 = w >> 4.
__device__ __forceinline__ uint32_t tc_q4_pair(uint32_t w, uint32_t w4, int e) {
  uint32_t v = __byte_perm(w, w4, (uint32_t)e | ((uint32_t)(4 + e) << 8));
  v = (v & 0x000F000Fu) | 0x43004300u;
  return tc_bits(__hsub2(tc_bf2(v), tc_bf2(0x43084308u)));
}

// Two Q8_0 codes (bytes e, e + 1 of w) as exact bf16.
__device__ __forceinline__ uint32_t tc_q8_pair(uint32_t w, int e) {
  const float a = (float)(int8_t)((w >> (8 * e)) & 0xFFu);
  const float b = (float)(int8_t)((w >> (8 * e + 8)) & 0xFFu);
  const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <int DT>
struct TcFmt {
  static constexpr int bb = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;  // bytes per block
  static constexpr int wpitch = kTcBpc * bb;                        // bytes per staged row
  static constexpr int wbytes = 128 * wpitch;                       // staged rows of a chunk
  static constexpr int xbytes = kTcMaxB * kTcXPitch;                // one input part of a chunk
  static constexpr int stage = wbytes + 2 * xbytes;                 // one buffer
};

template <int DT, bool DUAL>
__global__ void __launch_bounds__(kTcThreads, kTcMinBlocks) qmm_tc_kernel(TcParams p) {
  using F = TcFmt<DT>;
  constexpr int H2 = DUAL ? 2 : 1;
  constexpr int RPC = DUAL ? 64 : 128;  // rows of each matrix per CTA
  extern __shared__ __align__(128) unsigned char sm[];
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int h = DUAL ? warp >> 2 : 0, rt = DUAL ? warp & 3 : warp;
  const size_t r0 = (size_t)blockIdx.x * RPC;
  const int slice = blockIdx.y;
  const int kb0 = slice * p.slice_blocks, kb1 = min(p.nb, kb0 + p.slice_blocks);
  const int nch = (kb1 - kb0) / kTcBpc;
  const int NT = (p.B + 7) >> 3;
  const uint32_t sbase = smem_u32(sm);
  const size_t cols = (size_t)p.nb * kBlock;
  // stage chunk c (blocks kb0 + 4c ..) into buffer c mod kTcStages
  auto stage = [&](int c) {
    const uint32_t buf = sbase + (uint32_t)((c % kTcStages) * F::stage);
    const int kb = kb0 + c * kTcBpc;
    constexpr int ppr = F::wpitch / 16;  // 16-byte pieces per staged row
    for (int i = tid; i < 128 * ppr; i += kTcThreads) {
      const int lr = i / ppr, pc = i - lr * ppr;
      const int hh = DUAL ? lr >> 6 : 0;
      const size_t row = r0 + (DUAL ? (lr & 63) : lr);
      if (row >= p.rows) continue;
      const uint8_t* src = (hh ? p.w1 : p.w0) + (row * p.nb + kb) * F::bb + pc * 16;
      tc_cp16(buf + (uint32_t)(lr * F::wpitch + pc * 16), src);
    }
    for (int i = tid; i < 2 * p.B * 16; i += kTcThreads) {
      const int part = i / (p.B * 16), j = i - part * p.B * 16, b = j >> 4, pc = j & 15;
      const __nv_bfloat16* src = (part ? p.xl : p.xh) + (size_t)b * cols + (size_t)kb * kBlock + pc * 8;
      tc_cp16(buf + (uint32_t)(F::wbytes + part * F::xbytes + b * kTcXPitch + pc * 16), src);
    }
  };
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.0f;
  const int lrow = (DUAL ? 64 * h : 0) + 16 * rt + g;  // this lane's first staged row (+ 8: second)
  // ldmatrix row of this lane: matrix lane / 8 = (n-tile of the pair, k half)
  const int lm_n = 8 * ((lane >> 3) >> 1) + (lane & 7), lm_k = 8 * ((lane >> 3) & 1);
#pragma unroll
  for (int c = 0; c < kTcStages - 1; ++c) {
    if (c < nch) stage(c);
    tc_commit();
  }
  for (int c = 0; c < nch; ++c) {
    if (c + kTcStages - 1 < nch) stage(c + kTcStages - 1);
    tc_commit();
    tc_wait_stages();  // chunk c landed: at most kTcStages - 1 groups still pending
    __syncthreads();
    const uint32_t buf = sbase + (uint32_t)((c % kTcStages) * F::stage);
    const uint32_t wa = buf + (uint32_t)(lrow * F::wpitch), wb = wa + 8 * F::wpitch;
#pragma unroll
    for (int bl = 0; bl < kTcBpc; ++bl) {
      uint32_t a[2][4];  // A operand of k-steps 0, 1
      if (DT == MINQ_Q4_0) {
        const uint32_t x0 = tc_lds(wa + bl * F::bb + 4 + 4 * t), x1 = tc_lds(wb + bl * F::bb + 4 + 4 * t);
        const uint32_t x04 = x0 >> 4, x14 = x1 >> 4;
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          a[s][0] = tc_q4_pair(x0, x04, 2 * s);
          a[s][1] = tc_q4_pair(x1, x14, 2 * s);
          a[s][2] = tc_q4_pair(x0, x04, 2 * s + 1);
          a[s][3] = tc_q4_pair(x1, x14, 2 * s + 1);
        }
      } else {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const uint32_t x0 = tc_lds(wa + bl * F::bb + 4 + 4 * (2 * t + s));
          const uint32_t x1 = tc_lds(wb + bl * F::bb + 4 + 4 * (2 * t + s));
          a[s][0] = tc_q8_pair(x0, 0);
          a[s][1] = tc_q8_pair(x1, 0);
          a[s][2] = tc_q8_pair(x0, 2);
          a[s][3] = tc_q8_pair(x1, 2);
        }
      }
      const float d0 = __uint_as_float(tc_lds(wa + bl * F::bb));
      const float d1 = __uint_as_float(tc_lds(wb + bl * F::bb));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        if (2 * np >= NT) break;  // the same for the whole warp
        float c0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, c1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            uint32_t r[4];
            tc_ldsm4(buf + (uint32_t)(F::wbytes + part * F::xbytes) +
                         (uint32_t)((16 * np + lm_n) * kTcXPitch + (bl * kBlock + 16 * s + lm_k) * 2),
                     r);
            tc_mma(c0, a[s], r[0], r[1]);
            tc_mma(c1, a[s], r[2], r[3]);
          }
        acc[2 * np][0] = fmaf(d0, c0[0], acc[2 * np][0]);
        acc[2 * np][1] = fmaf(d0, c0[1], acc[2 * np][1]);
        acc[2 * np][2] = fmaf(d1, c0[2], acc[2 * np][2]);
        acc[2 * np][3] = fmaf(d1, c0[3], acc[2 * np][3]);
        acc[2 * np + 1][0] = fmaf(d0, c1[0], acc[2 * np + 1][0]);
        acc[2 * np + 1][1] = fmaf(d0, c1[1], acc[2 * np + 1][1]);
        acc[2 * np + 1][2] = fmaf(d1, c1[2], acc[2 * np + 1][2]);
        acc[2 * np + 1][3] = fmaf(d1, c1[3], acc[2 * np + 1][3]);
      }
    }
    __syncthreads();  // buffer c mod kTcStages is refilled from the next chunk on
  }
  tc_wait0();
  pdl_launch_dependents();
  // acc[n][i]: row r0 + 16 rt + g + 8 (i >> 1) of matrix h, input 8 n + 2 t + (i & 1)
  const size_t rowA = r0 + 16 * rt + g;
  if (p.S > 1 || !DUAL) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const size_t row = rowA + 8 * (i >> 1);
        const int b = 8 * n + 2 * t + (i & 1);
        if (n >= NT || b >= p.B || row >= p.rows) continue;
        if (p.S > 1) {
          p.part[(((size_t)slice * H2 + h) * p.B + b) * p.rows + row] = acc[n][i];
        } else {
          float y = acc[n][i];
          if (p.bias) y += p.bias[row];
          if (p.residual) y = p.residual[(size_t)b * p.y_stride + row] + y;
          p.y[(size_t)b * p.y_stride + row] = y;
        }
      }
    }
    return;
  }
  // dual, one slice: the up warps hand their sums to the gate warps
  float* xch = reinterpret_cast<float*>(sm);  // [4 row tiles][32 lanes][8][4]
  if (h == 1) {
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) xch[((rt * 32 + lane) * 8 + n) * 4 + i] = acc[n][i];
  }
  __syncthreads();
  if (h == 0) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const size_t row = rowA + 8 * (i >> 1);
        const int b = 8 * n + 2 * t + (i & 1);
        if (n >= NT || b >= p.B || row >= p.rows) continue;
        p.y[(size_t)b * p.y_stride + row] = silu(acc[n][i]) * xch[((rt * 32 + lane) * 8 + n) * 4 + i];
      }
    }
  }
}

// Sum of the S slices' partials in slice order, then the epilogue.
template <bool DUAL>
__global__ void __launch_bounds__(256) tc_reduce_kernel(TcParams p) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int H2 = DUAL ? 2 : 1;
  const size_t n = (size_t)p.B * p.rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / p.rows, row = i - b * p.rows;
    float v[H2];
#pragma unroll
    for (int hh = 0; hh < H2; ++hh) {
      v[hh] = 0.0f;
      for (int sl = 0; sl < p.S; ++sl) v[hh] += p.part[(((size_t)sl * H2 + hh) * p.B + b) * p.rows + row];
    }
    float y;
    if (DUAL) {
      y = silu(v[0]) * v[H2 - 1];
    } else {
      y = v[0];
      if (p.bias) y += p.bias[row];
      if (p.residual) y = p.residual[b * p.y_stride + row] + y;
    }
    p.y[b * p.y_stride + row] = y;
  }
}

template <int DT, bool DUAL>
minq_status tc_launch(const TcParams& p, unsigned tiles, cudaStream_t s) {
  const size_t smem = (size_t)kTcStages * TcFmt<DT>::stage;
  auto k = qmm_tc_kernel<DT, DUAL>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
  MINQ_CUDA_TRY(launch_k(k, dim3(tiles, (unsigned)p.S), dim3(kTcThreads), smem, s, p));
  if (p.S > 1) {
    const size_t n = (size_t)p.B * p.rows;
    const unsigned gr = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    MINQ_CUDA_TRY(launch_k(tc_reduce_kernel<DUAL>, dim3(gr), dim3(256), 0, s, p));
  }
  return MINQ_OK;
}

}  // namespace

bool qmatmul_tc_takes(int dtype, int cols, int B, size_t xp_floats) {
  return (dtype == MINQ_Q4_0 || dtype == MINQ_Q8_0) && B >= kQmmTcMinB && B <= kTcMaxB &&
         cols % kTcKc == 0 && xp_floats >= (size_t)B * cols;
}

minq_status launch_qmatmul_tc(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                              int B, const float* x, size_t x_stride, const float* norm_w, float eps,
                              float* xp, size_t xp_floats, const float* bias, const float* residual,
                              float* y, size_t y_stride, float* part, size_t part_floats,
                              cudaStream_t s) {
  if (!qmatmul_tc_takes(dtype, cols, B, xp_floats) || rows == 0)
    return fail(MINQ_ERR_ARG, "tensor-core batched matvec: dtype, shape or scratch");
  if ((uintptr_t)w0 % 16 || (w1 && (uintptr_t)w1 % 16))
    return fail(MINQ_ERR_ARG, "tensor-core batched matvec weights must be 16-byte aligned");
  __nv_bfloat16* xh = reinterpret_cast<__nv_bfloat16*>(xp);
  __nv_bfloat16* xl = xh + (size_t)B * cols;
  MINQ_CUDA_TRY(launch_k(tc_xprep_kernel,
                         dim3((unsigned)B, (unsigned)((cols + kTcPrepCols - 1) / kTcPrepCols)),
                         dim3(256), 0, s, x, x_stride, cols, norm_w, eps, xh, xl));
  TcParams p{};
  p.w0 = static_cast<const uint8_t*>(w0);
  p.w1 = static_cast<const uint8_t*>(w1);
  p.rows = rows;
  p.nb = cols / kBlock;
  p.B = B;
  p.xh = xh;
  p.xl = xl;
  p.bias = bias;
  p.residual = residual;
  p.y = y;
  p.y_stride = y_stride;
  p.part = part;
  // column slices of whole chunks: about two CTAs per SM, partials within
  // the workspace
  const int halves = w1 ? 2 : 1, rpc = w1 ? 64 : 128;
  const size_t tiles = (rows + rpc - 1) / rpc;
  const int nchunks = p.nb / kTcBpc;
  int S = (int)std::max<size_t>(1, (2 * 148 + tiles - 1) / tiles);
  S = std::min(S, nchunks);
  while (S > 1 && (!part || (size_t)S * halves * B * rows > part_floats)) --S;
  const int per = (nchunks + S - 1) / S;  // chunks per slice
  p.slice_blocks = per * kTcBpc;
  p.S = (nchunks + per - 1) / per;
  if (dtype == MINQ_Q4_0)
    return w1 ? tc_launch<MINQ_Q4_0, true>(p, (unsigned)tiles, s) : tc_launch<MINQ_Q4_0, false>(p, (unsigned)tiles, s);
  return w1 ? tc_launch<MINQ_Q8_0, true>(p, (unsigned)tiles, s) : tc_launch<MINQ_Q8_0, false>(p, (unsigned)tiles, s);
}

}  // namespace minq
