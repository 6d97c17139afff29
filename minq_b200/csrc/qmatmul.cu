// Batched projections for B independent sequences (one token each) or B
// tokens of one sequence on the CUDA cores (one quantized input, or f32
// weights; quantized projections of 2..64 inputs run on the tensor cores,
// qmatmul_tc.cu): Y[b] = W X[b] for Q8_0 / Q4_0 / f32 weights, with
// the input RMSNorm (tensor.rs:219-227) applied first and bias / residual /
// SwiGLU after, the weights read once for all B inputs.
//
// The rows are cut into tiles of 32 (one row per lane) and the columns into
// S slices (S chosen so the grid covers the GPU); a CTA of 8 warps takes one
// (row tile, column slice). Its warps split the inputs into groups of 8
// (TG = ceil(B / 8) groups) and the slice's blocks into 8 / TG interleaved
// parts; a lane reads its row's blocks straight from global memory (the
// lane's next block is in the same cache line, so L1 serves the rest of the
// line), decodes a block's 32 codes once and runs them against the 8 inputs
// of its group, which every lane of the warp reads at the same address (one
// broadcast load per 4 columns). Per block the arithmetic is the reference's
// (quantize.rs:252-280): sum = sum_k code_k x_k in f32, then acc += d * sum.
// Warp partials meet in shared memory (fixed order); with S > 1 the slices'
// partials go to a workspace and a second kernel sums them in slice order
// and applies the epilogue.
#include <algorithm>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "matvec_common.cuh"

namespace minq {

namespace {

constexpr int kQmmRows = 32;
constexpr int kQmmWarps = 8;
constexpr int kQmmChunk = 256;  // input columns staged in shared memory at a time

struct QmmParams {
  const void* w0;         // [rows][cols] blocks (or f32)
  const void* w1;         // dual: up rows, else null
  size_t rows;
  int cols;
  int B;
  const float* x;         // [B][x_stride] (normalised when the projection has a norm)
  size_t x_stride;
  int S;                  // column slices
  int slice_blocks;       // blocks per slice
  const float* bias;      // [rows] or null
  const float* residual;  // [B][y_stride] or null (may alias y)
  float* y;               // [B][y_stride]
  size_t y_stride;
  float* part;            // S > 1: [S][halves][B][rows]
};

template <int DT>
struct QmmFmt {
  static constexpr int bb = DT == MINQ_Q8_0 ? kQ8Bytes : DT == MINQ_Q4_0 ? kQ4Bytes : 128;
  static constexpr int bw = bb / 4;                            // words per block
  static constexpr int pitch = (kQmmChunk / kBlock) * bw + 1;  // odd: lanes hit distinct banks
};

// x_norm[b] = x[b] * inv_rms(x[b]) * w (tensor.rs:219-227), one CTA per input.
__global__ void __launch_bounds__(256) qmm_norm_kernel(const float* __restrict__ x, size_t x_stride,
                                                      int n, const float* __restrict__ w, float eps,
                                                      float* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[9];
  const float* row = x + (size_t)blockIdx.x * x_stride;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) v += red[k];
    red[8] = 1.0f / sqrtf(v / (float)n + eps);
  }
  __syncthreads();
  const float inv = red[8];
  float* o = out + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = row[i] * inv * w[i];
}

// 32 weights of one block (shared-memory words) as floats (code - 8 for
// Q4_0, the i8 code for Q8_0, the f32 values), and the block scale (1 for
// f32).
template <int DT>
__device__ __forceinline__ float qmm_block(const uint32_t* w, float (&c)[32]) {
  if (DT == MINQ_Q4_0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t v = w[1 + q];
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // byte 4q + e: columns 8q + 2e (low nibble), + 1 (high)
        const int byte = (int)((v >> (8 * e)) & 0xFFu);
        c[8 * q + 2 * e] = (float)((byte & 15) - 8);
        c[8 * q + 2 * e + 1] = (float)((byte >> 4) - 8);
      }
    }
    return __uint_as_float(w[0]);
  } else if (DT == MINQ_Q8_0) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t v = w[1 + q];
#pragma unroll
      for (int e = 0; e < 4; ++e) c[4 * q + e] = (float)(int8_t)((v >> (8 * e)) & 0xFFu);
    }
    return __uint_as_float(w[0]);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) c[k] = __uint_as_float(w[k]);
    return 1.0f;
  }
}

template <int DT, bool DUAL>
__global__ void __launch_bounds__(kQmmRows* kQmmWarps) qmatmul_kernel(QmmParams p) {
  constexpr int H2 = DUAL ? 2 : 1;
  __shared__ float red[kQmmWarps][H2][8][kQmmRows];  // warp partials
  extern __shared__ __align__(16) float xs[];         // [B][kQmmChunk] inputs of a chunk,
  uint32_t* wsm = reinterpret_cast<uint32_t*>(xs + (size_t)p.B * kQmmChunk);  // then [H2][32][pitch]
  using F = QmmFmt<DT>;
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int TG = (p.B + 7) >> 3, BS = kQmmWarps / TG;  // input groups, block parts
  const int grp = warp / BS, part = warp - grp * BS;
  const size_t r0 = (size_t)blockIdx.x * kQmmRows;
  const int slice = blockIdx.y;
  const int nb = p.cols / kBlock;
  const int kb0 = slice * p.slice_blocks, kb1 = min(nb, kb0 + p.slice_blocks);
  const size_t r = r0 + lane;
  const bool has_row = r < p.rows && grp < TG;
  const int b0 = grp * 8, nbk = min(8, p.B - b0);
  float acc[H2][8];
#pragma unroll
  for (int h = 0; h < H2; ++h)
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[h][t] = 0.0f;
  for (int cb = kb0; cb < kb1; cb += kQmmChunk / kBlock) {  // chunks of 256 columns
    const int cbk = min(kQmmChunk / kBlock, kb1 - cb), nq = cbk * kBlock / 4;
    __syncthreads();  // the previous chunk is consumed
    for (int i = tid; i < p.B * nq; i += blockDim.x) {
      const int b = i / nq, q = i - b * nq;
      reinterpret_cast<float4*>(xs + (size_t)b * kQmmChunk)[q] =
          __ldg(reinterpret_cast<const float4*>(p.x + (size_t)b * p.x_stride + cb * kBlock) + q);
    }
    {  // the tile's rows of this chunk, coalesced word loads into the padded layout
      const int cw = cbk * F::bw, nrows = (int)min((size_t)kQmmRows, p.rows - r0);
      for (int h = 0; h < H2; ++h) {
        const uint32_t* src = static_cast<const uint32_t*>(h ? p.w1 : p.w0) +
                              (r0 * (size_t)nb + cb) * F::bw;
        uint32_t* dst = wsm + (size_t)h * kQmmRows * F::pitch;
        for (int i = tid; i < nrows * cw; i += blockDim.x) {
          const int rr = i / cw, w = i - rr * cw;
          dst[rr * F::pitch + w] = __ldg(src + (size_t)rr * nb * F::bw + w);
        }
      }
    }
    __syncthreads();
    if (!has_row) continue;
    for (int kb = cb + part; kb < cb + cbk; kb += BS) {
#pragma unroll
      for (int h = 0; h < H2; ++h) {
        float c[32];
        const float d =
            qmm_block<DT>(wsm + ((size_t)h * kQmmRows + lane) * F::pitch + (kb - cb) * F::bw, c);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < nbk) {
            const float4* xv =
                reinterpret_cast<const float4*>(xs + (size_t)(b0 + t) * kQmmChunk + (kb - cb) * kBlock);
            float sum = 0.0f;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 v = xv[q];
              sum = fmaf(c[4 * q], v.x, sum);
              sum = fmaf(c[4 * q + 1], v.y, sum);
              sum = fmaf(c[4 * q + 2], v.z, sum);
              sum = fmaf(c[4 * q + 3], v.w, sum);
            }
            acc[h][t] = DT == MINQ_F32 ? acc[h][t] + sum : fmaf(d, sum, acc[h][t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < H2; ++h)
#pragma unroll
    for (int t = 0; t < 8; ++t) red[warp][h][t][lane] = acc[h][t];
  __syncthreads();
  pdl_launch_dependents();
  // one thread per (input, row): sum the block parts in order
  for (int i = tid; i < p.B * kQmmRows; i += blockDim.x) {
    const int b = i / kQmmRows, ln = i - b * kQmmRows;
    const size_t row = r0 + ln;
    if (row >= p.rows) continue;
    const int g = b >> 3, t = b & 7;
    float v[H2];
#pragma unroll
    for (int h = 0; h < H2; ++h) {
      v[h] = 0.0f;
      for (int pp = 0; pp < BS; ++pp) v[h] += red[g * BS + pp][h][t][ln];
    }
    if (p.S > 1) {
#pragma unroll
      for (int h = 0; h < H2; ++h)
        p.part[(((size_t)slice * H2 + h) * p.B + b) * p.rows + row] = v[h];
      continue;
    }
    float y;
    if (DUAL) {
      y = silu(v[0]) * v[H2 - 1];
    } else {
      y = v[0];
      if (p.bias) y += p.bias[row];
      if (p.residual) y = p.residual[(size_t)b * p.y_stride + row] + y;
    }
    p.y[(size_t)b * p.y_stride + row] = y;
  }
}

// Sum of the S slices' partials in slice order, then the epilogue.
template <bool DUAL>
__global__ void __launch_bounds__(256) qmm_reduce_kernel(QmmParams p) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int H2 = DUAL ? 2 : 1;
  const size_t n = (size_t)p.B * p.rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / p.rows, row = i - b * p.rows;
    float v[H2];
#pragma unroll
    for (int h = 0; h < H2; ++h) {
      v[h] = 0.0f;
      for (int sl = 0; sl < p.S; ++sl) v[h] += p.part[(((size_t)sl * H2 + h) * p.B + b) * p.rows + row];
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

__global__ void embed_batch_kernel(const float* __restrict__ embed, const uint32_t* tok,
                                   size_t vocab, int hidden, float* __restrict__ x) {
  pdl_wait();
  pdl_launch_dependents();
  uint32_t t = tok[blockIdx.y];
  if (t >= vocab) t = 0;  // host validates tokens; never read out of bounds
  const float* row = embed + (size_t)t * hidden;
  float* out = x + (size_t)blockIdx.y * hidden;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
    out[i] = row[i];
}

// argmax of each row of x [B][n] (sampler.rs:10-17: f32::total_cmp order,
// ties to the lowest index): CTA (b, j) packs the best of part j of row b
// (kArgParts parts, eight loads in flight per thread), then one warp per row
// takes the best of the parts.
constexpr int kArgParts = 32;
__global__ void __launch_bounds__(256) argmax_rows_part_kernel(const float* __restrict__ x, size_t n,
                                                               unsigned long long* part) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ unsigned long long red[8];
  const float* row = x + (size_t)blockIdx.x * n;
  const size_t c0 = n * blockIdx.y / kArgParts, c1 = n * (blockIdx.y + 1) / kArgParts;
  unsigned long long best = 0;
#pragma unroll 8
  for (size_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const unsigned long long pk = argmax_pack(row[i], (uint32_t)i);
    best = pk > best ? pk : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    part[(size_t)blockIdx.x * kArgParts + blockIdx.y] = best;
  }
}

__global__ void __launch_bounds__(32) argmax_rows_final_kernel(const unsigned long long* part,
                                                              uint32_t* out) {
  pdl_wait();
  pdl_launch_dependents();
  unsigned long long best = part[(size_t)blockIdx.x * kArgParts + threadIdx.x];
  best = warp_max_u64(best);
  if (threadIdx.x == 0) out[blockIdx.x] = argmax_unpack_index(best);
}

template <int DT, bool DUAL>
minq_status qmm_launch(QmmParams p, cudaStream_t s) {
  const unsigned tiles = (unsigned)((p.rows + kQmmRows - 1) / kQmmRows);
  const size_t smem = (size_t)p.B * kQmmChunk * 4 +
                      (DUAL ? 2 : 1) * (size_t)kQmmRows * QmmFmt<DT>::pitch * 4;
  auto k = qmatmul_kernel<DT, DUAL>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
  MINQ_CUDA_TRY(launch_k(k, dim3(tiles, (unsigned)p.S), dim3(kQmmRows * kQmmWarps), smem, s, p));
  if (p.S > 1) {
    const size_t n = (size_t)p.B * p.rows;
    const unsigned g = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    MINQ_CUDA_TRY(launch_k(qmm_reduce_kernel<DUAL>, dim3(g), dim3(256), 0, s, p));
  }
  return MINQ_OK;
}

}  // namespace

// MINQ_TCGEN05=0 in the environment selects the mma.sync kernel for the
// tensor-core batched projections (comparison runs); default: tcgen05.
static bool umma_enabled() {
  static const bool on = [] {
    const char* e = getenv("MINQ_TCGEN05");
    return !(e && e[0] == '0');
  }();
  return on;
}

minq_status launch_qmatmul(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                           int B, const float* x, size_t x_stride, const float* norm_w, float eps,
                           float* xn_scratch, size_t xn_floats, const float* bias,
                           const float* residual, float* y, size_t y_stride, float* part,
                           size_t part_floats, cudaStream_t s) {
  if (B < 1 || B > kQmmMaxB) return fail(MINQ_ERR_ARG, "batched matvec takes 1..64 inputs");
  if (B >= kQmmTcMinB && xn_scratch && umma_enabled() && qmatmul_umma_takes(dtype, cols, B, xn_floats))
    return launch_qmatmul_umma(dtype, w0, w1, rows, cols, B, x, x_stride, norm_w, eps, xn_scratch,
                               xn_floats, bias, residual, y, y_stride, part, part_floats, s);
  if (xn_scratch && qmatmul_tc_takes(dtype, cols, B, xn_floats))
    return launch_qmatmul_tc(dtype, w0, w1, rows, cols, B, x, x_stride, norm_w, eps, xn_scratch,
                             xn_floats, bias, residual, y, y_stride, part, part_floats, s);
  if (cols % kBlock != 0 || rows == 0) return fail(MINQ_ERR_SHAPE, "batched matvec shape");
  if (dtype != MINQ_Q8_0 && dtype != MINQ_Q4_0 && dtype != MINQ_F32)
    return fail(MINQ_ERR_ARG, "batched matvec dtype");
  if (w1 && dtype == MINQ_F32) return fail(MINQ_ERR_ARG, "dual batched matvec needs blocks");
  if (x_stride % 4 != 0 || (uintptr_t)x % 16 != 0 || (dtype == MINQ_F32 && (uintptr_t)w0 % 16))
    return fail(MINQ_ERR_ARG, "batched matvec inputs must be 16-byte aligned");
  if (norm_w) {  // normalised inputs first, contiguous [B][cols]
    if (!xn_scratch) return fail(MINQ_ERR_ARG, "batched RMSNorm needs a scratch buffer");
    MINQ_CUDA_TRY(launch_k(qmm_norm_kernel, dim3((unsigned)B), dim3(256), 0, s, x, x_stride, cols,
                           norm_w, eps, xn_scratch));
    x = xn_scratch;
    x_stride = (size_t)cols;
  }
  if (dtype == MINQ_F32 && !bias && !residual && f32_gemm_takes(B, cols, w0, x, x_stride))
    return launch_f32_gemm(static_cast<const float*>(w0), rows, cols, x, x_stride, B, y, y_stride,
                           s);
  QmmParams p{};
  p.w0 = w0;
  p.w1 = w1;
  p.rows = rows;
  p.cols = cols;
  p.B = B;
  p.x = x;
  p.x_stride = x_stride;
  p.bias = bias;
  p.residual = residual;
  p.y = y;
  p.y_stride = y_stride;
  p.part = part;
  // column slices: enough CTAs for ~4 per SM, at least 8 blocks per slice,
  // and the partials within the workspace
  const int nb = cols / kBlock, halves = w1 ? 2 : 1;
  const size_t tiles = (rows + kQmmRows - 1) / kQmmRows;
  int S = (int)std::max<size_t>(1, (4 * 148 + tiles - 1) / tiles);
  S = std::min(S, std::max(1, nb / 8));
  while (S > 1 && (size_t)S * halves * B * rows > part_floats) --S;
  if (S > 1 && !part) S = 1;
  p.S = S;
  p.slice_blocks = (nb + S - 1) / S;
  if (dtype == MINQ_Q4_0) return w1 ? qmm_launch<MINQ_Q4_0, true>(p, s) : qmm_launch<MINQ_Q4_0, false>(p, s);
  if (dtype == MINQ_Q8_0) return w1 ? qmm_launch<MINQ_Q8_0, true>(p, s) : qmm_launch<MINQ_Q8_0, false>(p, s);
  return qmm_launch<MINQ_F32, false>(p, s);
}

minq_status launch_embed_batch(const float* embed, const uint32_t* d_tok, size_t vocab, int hidden,
                               int B, float* x, cudaStream_t s) {
  const unsigned gx = (unsigned)std::min(8, (hidden + 255) / 256);
  MINQ_CUDA_TRY(launch_k(embed_batch_kernel, dim3(gx, (unsigned)B), dim3(256), 0, s, embed, d_tok,
                         vocab, hidden, x));
  return MINQ_OK;
}

minq_status launch_argmax_rows(const float* x, size_t n, int B, uint32_t* out,
                               unsigned long long* scratch, cudaStream_t s) {
  static_assert(kArgParts == 32, "one warp reduces the parts");
  MINQ_CUDA_TRY(launch_k(argmax_rows_part_kernel, dim3((unsigned)B, kArgParts), dim3(256), 0, s, x,
                         n, scratch));
  MINQ_CUDA_TRY(launch_k(argmax_rows_final_kernel, dim3((unsigned)B), dim3(32), 0, s,
                         (const unsigned long long*)scratch, out));
  return MINQ_OK;
}

}  // namespace minq
