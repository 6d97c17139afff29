// Batch-1 matvec kernels (HBM-bound, CUDA cores) for the block-quantized
// weights of quantize.rs and the dense f32 lm_head of tensor.rs, and the
// launch dispatch.
//
// QuantizedTensor::matvec (quantize.rs:215-280):
//   * rows whose byte length is a multiple of 16 (cols % 128 == 0, every
//     benchmark shape) go to the TMA-fed kernel of qmatvec_tma.cu;
//   * other shapes use the generic kernel below: a warp sweeps R rows in
//     chunks of 8 blocks (256 columns); lane = 4*block + sub owns 8
//     consecutive columns of one block, so its codes are one 32-bit word
//     (Q4_0) or two (Q8_0) at a 4-byte-aligned offset and its 8 x-values are
//     two float4s of a shared-memory copy of x; when there are too few row
//     groups, KS warps split the columns and reduce through shared memory.
// Both paths: the weight stays in the reference's AoS block layout, codes
// become exact floats (byte permute into the mantissa of 2^23, subtract),
// the block scale is applied once per block (acc += d * partial, as the
// reference does), x is staged once per CTA with the optional RMSNorm
// (tensor.rs:219-227) applied on the way, and the epilogue adds the bias
// (model.rs:282-290), the residual (model.rs:305,314) or forms the SwiGLU
// product silu(gate)*up (model.rs:309-312) over a gate/up row pair.
#include <cuda.h>

#include <algorithm>

#include "kernels.h"
#include "ktimer.h"
#include "matvec_common.cuh"
#include "pipeline.cuh"

namespace minq {

minq_status launch_qmatvec_tma(const MatvecParams& p, int dtype, const QmvPlan& t,
                               const CUtensorMap* m0, const CUtensorMap* m1, cudaStream_t s);

// R = rows per row group; DUAL = rows come in (gate, up) pairs.
template <int DT, int R, bool DUAL>
__global__ void __launch_bounds__(256) qmatvec_kernel(MatvecParams p) {
  extern __shared__ float smem[];
  float* red = smem;              // [8 warps * NR] + 33
  float* xs = smem + 8 * 8 + 40;  // [cols]
  constexpr int NR = DUAL ? 2 * R : R;
  constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  pdl_wait();
  pdl_launch_dependents();
  stage_x(p, xs, red + 8 * NR);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ks = p.ks;
  const int groups_per_cta = 8 / ks;
  const int gslot = warp / ks, kslot = warp % ks;
  const int nb = p.cols / kBlock;
  const int nchunks = (nb + 7) >> 3;
  const size_t row_bytes = (size_t)nb * BB;
  const int bi = lane >> 2, sub = lane & 3;
  const size_t ngroups = (p.rows + R - 1) / R;

  for (size_t g0 = (size_t)blockIdx.x * groups_per_cta; g0 < ngroups;
       g0 += (size_t)gridDim.x * groups_per_cta) {
    const size_t g = g0 + gslot;
    const size_t r0 = g * R;
    float acc[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) acc[i] = 0.0f;
    if (g < ngroups) {
      const uint8_t* rowp[NR];
      bool ok[NR];
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        size_t r = r0 + (DUAL ? (i >> 1) : i);
        ok[i] = r < p.rows;
        const uint8_t* base = (DUAL && (i & 1)) ? p.w1 : p.w0;
        rowp[i] = base + (ok[i] ? r : 0) * row_bytes;
      }
#pragma unroll 2
      for (int c = kslot; c < nchunks; c += ks) {
        const int b = c * 8 + bi;
        if (b < nb) {
          const float4 xa = *reinterpret_cast<const float4*>(xs + 32 * b + 8 * sub);
          const float4 xb = *reinterpret_cast<const float4*>(xs + 32 * b + 8 * sub + 4);
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            if (ok[i]) {
              const uint8_t* blk = rowp[i] + (size_t)b * BB;
              const float d = __ldg(reinterpret_cast<const float*>(blk));
              acc[i] = fmaf(d, lane_dot<DT>(blk, sub, xa, xb), acc[i]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) acc[i] = warp_sum(acc[i]);
    if (ks > 1) {
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < NR; ++i) red[warp * NR + i] = acc[i];
      }
      __syncthreads();
      if (kslot == 0) {
        for (int w = 1; w < ks; ++w) {
#pragma unroll
          for (int i = 0; i < NR; ++i) acc[i] += red[(warp + w) * NR + i];
        }
      }
    }
    if (g < ngroups && kslot == 0 && lane < R) {
      float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (lane == r) {
          v0 = DUAL ? acc[2 * r] : acc[r];
          v1 = DUAL ? acc[2 * r + 1] : 0.0f;
        }
      }
      const size_t r = r0 + lane;
      if (r < p.rows) {
        float v;
        if (DUAL) {
          v = silu(v0) * v1;
        } else {
          v = v0;
          if (p.bias) v += p.bias[r];
          if (p.residual) v = p.residual[r] + v;
        }
        p.y[r] = v;
      }
    }
    if (ks > 1) __syncthreads();
  }
}

// Dense f32 matvec (tensor.rs:181-192), the tied lm_head: R rows per warp,
// float4 streaming loads of W (evict-first) with the 32 lanes covering 128
// consecutive columns per step; x (optionally RMS-normalised) in shared
// memory. Fused argmax: each CTA writes its best (value, index), packed so
// that an integer max reproduces f32::total_cmp with ties to the lowest
// index (sampler.rs:10-17).
template <int R>
__global__ void __launch_bounds__(256) f32_matvec_kernel(MatvecParams p) {
  extern __shared__ float smem[];
  float* red = smem;
  float* xs = smem + 8 * 8 + 40;
  pdl_wait();
  pdl_launch_dependents();
  stage_x(p, xs, red + 8 * R);
  __shared__ unsigned long long best_s[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* W = reinterpret_cast<const float*>(p.w0);
  const int cols = p.cols;
  const int nvec = cols >> 2;  // cols % 4 == 0 (checked on the host)
  const size_t ngroups = (p.rows + R - 1) / R;
  unsigned long long best = 0;
  for (size_t g = (size_t)blockIdx.x * 8 + warp; g < ngroups; g += (size_t)gridDim.x * 8) {
    const size_t r0 = g * R;
    float acc[R];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = 0.0f;
    const float4* rowp[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      size_t r = r0 + i < p.rows ? r0 + i : p.rows - 1;
      rowp[i] = reinterpret_cast<const float4*>(W + r * (size_t)cols);
    }
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      const float4 xv = reinterpret_cast<const float4*>(xs)[v];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const float4 wv = __ldcs(rowp[i] + v);
        acc[i] = fmaf(wv.x, xv.x, acc[i]);
        acc[i] = fmaf(wv.y, xv.y, acc[i]);
        acc[i] = fmaf(wv.z, xv.z, acc[i]);
        acc[i] = fmaf(wv.w, xv.w, acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = warp_sum(acc[i]);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const size_t r = r0 + i;
      if (r < p.rows) {
        if (lane == i) p.y[r] = acc[i];
        unsigned long long pk = argmax_pack(acc[i], (uint32_t)r);
        best = pk > best ? pk : best;
      }
    }
  }
  if (p.argmax_part) {
    best = warp_max_u64(best);
    if (lane == 0) best_s[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = best_s[0];
      for (int w = 1; w < 8; ++w) b = best_s[w] > b ? best_s[w] : b;
      p.argmax_part[blockIdx.x] = b;
    }
  }
}

// Reduce per-CTA packed argmax partials to one index.
__global__ void argmax_final_kernel(const unsigned long long* part, int n, uint32_t* out) {
  pdl_wait();
  pdl_launch_dependents();
  unsigned long long b = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) b = part[i] > b ? part[i] : b;
  b = warp_max_u64(b);
  __shared__ unsigned long long s[32];
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x < 32) {
    b = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0;
    b = warp_max_u64(b);
    if (threadIdx.x == 0) *out = argmax_unpack_index(b);
  }
}

// Standalone argmax over a logits vector (sampler.rs:10-17).
__global__ void argmax_partial_kernel(const float* x, size_t n, unsigned long long* part) {
  pdl_wait();
  pdl_launch_dependents();
  unsigned long long b = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    unsigned long long pk = argmax_pack(x[i], (uint32_t)i);
    b = pk > b ? pk : b;
  }
  b = warp_max_u64(b);
  __shared__ unsigned long long s[32];
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x < 32) {
    b = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0;
    b = warp_max_u64(b);
    if (threadIdx.x == 0) part[blockIdx.x] = b;
  }
}

// ---------------------------------------------------------------------------
// Host launchers.

static size_t xs_smem_bytes(int cols) { return (size_t)(8 * 8 + 40 + cols) * sizeof(float); }

template <typename K>
static minq_status set_smem(K kernel, size_t bytes) {
  return ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), bytes);
}

// Pick the column split so that enough warps are resident to keep HBM busy.
static int choose_ks(size_t ngroups, int nchunks) {
  const size_t target = (size_t)sm_count() * 16;
  int ks = 1;
  while (ks < 8 && ngroups * ks < target && ks * 2 <= nchunks) ks *= 2;
  return ks;
}

static unsigned persistent_grid(size_t ctas_needed, size_t smem_bytes) {
  size_t per_sm = smem_bytes > 0 ? (200 * 1024) / smem_bytes : 8;
  if (per_sm > 8) per_sm = 8;
  if (per_sm < 1) per_sm = 1;
  size_t cap = (size_t)sm_count() * per_sm;
  size_t g = ctas_needed < cap ? ctas_needed : cap;
  return (unsigned)(g ? g : 1);
}

bool qmatvec_uses_tma(int cols, const void* w0, const void* w1, const float* x,
                      const float* norm_w) {
  return cols % 128 == 0 && (uintptr_t)w0 % 16 == 0 && (!w1 || (uintptr_t)w1 % 16 == 0) &&
         (uintptr_t)x % 16 == 0 && (!norm_w || (uintptr_t)norm_w % 16 == 0);
}

// `m0` / `m1`: optional pre-encoded tensor maps for the TMA path (encoded
// with plan_qmatvec_tma's nr for this shape).
minq_status launch_qmatvec(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                           const float* x, const float* norm_w, float eps, const float* bias,
                           const float* residual, float* y, cudaStream_t s,
                           const CUtensorMap* m0, const CUtensorMap* m1) {
  if (rows == 0) return MINQ_OK;
  MatvecParams p{};
  p.w0 = (const uint8_t*)w0;
  p.w1 = (const uint8_t*)w1;
  p.rows = rows;
  p.cols = cols;
  p.x = x;
  p.norm_w = norm_w;
  p.eps = eps;
  p.bias = bias;
  p.residual = residual;
  p.y = y;
  p.status = device_status_word();
  const bool dual = w1 != nullptr;
  const double wbytes = (double)rows * (cols / kBlock) * block_bytes(dtype) * (dual ? 2 : 1);
  ScopedKTimer timer(KF_QMATVEC, s,
                     wbytes + 4.0 * cols * (norm_w ? 2 : 1) +
                         4.0 * rows * (1 + (bias ? 1 : 0) + (residual ? 1 : 0)));
  if (qmatvec_uses_tma(cols, w0, w1, x, norm_w)) {
    const QmvPlan t = plan_qmatvec_tma(dtype, dual, rows, cols, norm_w != nullptr);
    return launch_qmatvec_tma(p, dtype, t, m0, m1, s);
  }
  constexpr int R_SINGLE = 4, R_DUAL = 2;
  const int R = dual ? R_DUAL : R_SINGLE;
  const size_t ngroups = (rows + R - 1) / R;
  const int nchunks = (cols / kBlock + 7) / 8;
  p.ks = choose_ks(ngroups, nchunks);
  const size_t smem = xs_smem_bytes(cols);
  const size_t ctas = (ngroups + (8 / p.ks) - 1) / (8 / p.ks);
  const unsigned grid = persistent_grid(ctas, smem);
#define MINQ_QMV(DT, RR, DU)             \
  do {                                   \
    auto k = qmatvec_kernel<DT, RR, DU>; \
    MINQ_TRY(set_smem(k, smem));         \
    MINQ_CUDA_TRY(launch_k(k, dim3(grid), dim3(256), smem, s, p)); \
  } while (0)
  if (dtype == MINQ_Q8_0) {
    if (dual) MINQ_QMV(MINQ_Q8_0, R_DUAL, true);
    else MINQ_QMV(MINQ_Q8_0, R_SINGLE, false);
  } else {
    if (dual) MINQ_QMV(MINQ_Q4_0, R_DUAL, true);
    else MINQ_QMV(MINQ_Q4_0, R_SINGLE, false);
  }
#undef MINQ_QMV
  MINQ_LAUNCH_CHECK("qmatvec_kernel");
  return MINQ_OK;
}

// Returns the number of argmax partials written (grid size) via *n_part.
minq_status launch_f32_matvec(const float* w, size_t rows, int cols, const float* x,
                              const float* norm_w, float eps, float* y,
                              unsigned long long* argmax_part, int* n_part, cudaStream_t s) {
  if (rows == 0) return MINQ_OK;
  MatvecParams p{};
  p.w0 = (const uint8_t*)w;
  p.rows = rows;
  p.cols = cols;
  p.x = x;
  p.norm_w = norm_w;
  p.eps = eps;
  p.y = y;
  p.argmax_part = argmax_part;
  constexpr int R = 4;
  const size_t ngroups = (rows + R - 1) / R;
  const size_t smem = xs_smem_bytes(cols);
  unsigned grid = persistent_grid((ngroups + 7) / 8, smem);
  if (n_part) {
    if ((int)grid > *n_part) grid = (unsigned)*n_part;  // capacity of the partials buffer
    *n_part = (int)grid;
  }
  auto k = f32_matvec_kernel<R>;
  MINQ_TRY(set_smem(k, smem));
  ScopedKTimer timer(KF_F32_MATVEC, s,
                     4.0 * rows * cols + 4.0 * cols * (norm_w ? 2 : 1) + 4.0 * rows);
  MINQ_CUDA_TRY(launch_k(k, dim3(grid), dim3(256), smem, s, p));
  MINQ_LAUNCH_CHECK("f32_matvec_kernel");
  return MINQ_OK;
}

minq_status launch_argmax_final(const unsigned long long* part, int n, uint32_t* out,
                                cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(argmax_final_kernel, dim3(1), dim3(256), 0, s, part, n, out));
  MINQ_LAUNCH_CHECK("argmax_final_kernel");
  return MINQ_OK;
}

minq_status launch_argmax(const float* x, size_t n, unsigned long long* part, int n_part,
                          uint32_t* out, cudaStream_t s) {
  size_t g = (n + 255) / 256;
  if (g > (size_t)n_part) g = n_part;
  if (g == 0) g = 1;
  MINQ_CUDA_TRY(launch_k(argmax_partial_kernel, dim3((unsigned)g), dim3(256), 0, s, x, n, part));
  MINQ_LAUNCH_CHECK("argmax_partial_kernel");
  return launch_argmax_final(part, (int)g, out, s);
}

// Largest number of per-CTA argmax partials any launch above can produce.
int argmax_parts_capacity() { return sm_count() * 8 + 8; }

}  // namespace minq
