// Dense f32 weights against many inputs: Y[b][r] = sum_k W[r][k] X[b][k] for
// 32..64 inputs. This is tensor::matvec (tensor.rs:181-192) once per input:
// the tied f32 lm_head (model.rs:562-565) over the scored positions of a
// perplexity chunk (ppl.rs:75-82) and over a batch of sequences. The weights
// are f32, so the product stays on the CUDA cores in f32 (a tensor-core
// TF32 product would round the table to 11 bits).
//
// A CTA owns 128 weight rows and all (up to 64) inputs, so the table is read
// from HBM exactly once per call. Both operands are K-major in memory and are
// staged as they lie, 32 columns at a time, into a three-stage cp.async ring
// (rows padded to 36 floats: the 8 lanes of a 16-byte load phase hit 8
// distinct 4-bank groups). Thread (lane, warp) accumulates rows lane + 32 i
// (i < 4) against inputs warp + 8 j (j < 8): per 4 columns it loads four
// 16-byte row pieces (distinct per lane) and eight input pieces (the same
// address across the warp: broadcasts) for 128 FMAs. Each output is one
// sequential f32 sum over k.
#include "common.cuh"
#include "kernels.h"
#include "pipeline.cuh"

namespace minq {

namespace {

constexpr int kFgRows = 128;           // weight rows per CTA
constexpr int kFgB = 64;               // inputs per CTA (all of them)
constexpr int kFgK = 32;               // columns per stage
constexpr int kFgPitch = kFgK + 4;     // floats per staged row
constexpr int kFgStages = 3;
constexpr int kFgThreads = 256;
constexpr size_t kFgSmem =
    sizeof(float) * (size_t)kFgStages * (kFgRows + kFgB) * kFgPitch;  // 82,944 B

__device__ __forceinline__ void fg_cp16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void fg_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void fg_wait_all_but_one() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kFgStages - 2) : "memory");
}

__global__ void __launch_bounds__(kFgThreads, 2)
    f32_gemm_kernel(const float* __restrict__ W, size_t rows, int K, const float* __restrict__ X,
                    size_t x_stride, int B, float* __restrict__ Y, size_t y_stride) {
  extern __shared__ __align__(16) float fg_smem[];
  float* Ws = fg_smem;                                    // [stage][128][pitch]
  float* Xs = Ws + (size_t)kFgStages * kFgRows * kFgPitch;  // [stage][64][pitch]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t r0 = (size_t)blockIdx.x * kFgRows;
  const int nk = K / kFgK;
  pdl_wait();  // X may come from the previous kernel on the stream
  // Stage kt: 128 rows x 8 pieces of 16 bytes (4 per thread) and 64 inputs
  // x 8 pieces (2 per thread). Rows past the table and inputs past B reread
  // the last valid one; their sums are never stored.
  auto load_stage = [&](int st, int kt) {
    const int k0 = kt * kFgK;
    float* ws = Ws + (size_t)st * kFgRows * kFgPitch;
    float* xs = Xs + (size_t)st * kFgB * kFgPitch;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int piece = tid + i * kFgThreads;
      const int row = piece >> 3, c4 = piece & 7;
      const size_t gr = r0 + row < rows ? r0 + row : rows - 1;
      fg_cp16(ws + row * kFgPitch + 4 * c4, W + gr * (size_t)K + k0 + 4 * c4);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int piece = tid + i * kFgThreads;
      const int b = piece >> 3, c4 = piece & 7;
      const int gb = b < B ? b : B - 1;
      fg_cp16(xs + b * kFgPitch + 4 * c4, X + (size_t)gb * x_stride + k0 + 4 * c4);
    }
  };
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
#pragma unroll
  for (int s = 0; s < kFgStages - 1; ++s) {
    if (s < nk) load_stage(s, s);
    fg_commit();
  }
  for (int kt = 0; kt < nk; ++kt) {
    // stage kt has landed for this thread; the barrier makes every thread's
    // copies visible and retires the stage refilled next (read in kt - 1)
    fg_wait_all_but_one();
    __syncthreads();
    const int nxt = kt + kFgStages - 1;
    if (nxt < nk) load_stage(nxt % kFgStages, nxt);
    fg_commit();
    const float* ws = Ws + (size_t)(kt % kFgStages) * kFgRows * kFgPitch + lane * kFgPitch;
    const float* xs = Xs + (size_t)(kt % kFgStages) * kFgB * kFgPitch + warp * kFgPitch;
#pragma unroll
    for (int kk = 0; kk < kFgK; kk += 4) {
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = *reinterpret_cast<const float4*>(ws + 32 * i * kFgPitch + kk);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 b = *reinterpret_cast<const float4*>(xs + 8 * j * kFgPitch + kk);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float t = acc[i][j];
          t = fmaf(a[i].x, b.x, t);
          t = fmaf(a[i].y, b.y, t);
          t = fmaf(a[i].z, b.z, t);
          t = fmaf(a[i].w, b.w, t);
          acc[i][j] = t;
        }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  pdl_launch_dependents();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int b = warp + 8 * j;
    if (b >= B) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const size_t r = r0 + lane + 32 * i;
      if (r < rows) Y[(size_t)b * y_stride + r] = acc[i][j];
    }
  }
}

}  // namespace

bool f32_gemm_takes(int B, int cols, const void* w, const float* x, size_t x_stride) {
  return B >= kF32GemmMinB && B <= kFgB && cols > 0 && cols % kFgK == 0 && x_stride % 4 == 0 &&
         (uintptr_t)w % 16 == 0 && (uintptr_t)x % 16 == 0;
}

minq_status launch_f32_gemm(const float* w, size_t rows, int cols, const float* x, size_t x_stride,
                            int B, float* y, size_t y_stride, cudaStream_t s) {
  if (!f32_gemm_takes(B, cols, w, x, x_stride))
    return fail(MINQ_ERR_ARG, "f32 GEMM: 32..64 inputs, 32-column multiples, 16-byte alignment");
  if (rows == 0) return MINQ_OK;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(f32_gemm_kernel), kFgSmem));
  const size_t grid = (rows + kFgRows - 1) / kFgRows;
  if (grid > 0x7fffffffu) return fail(MINQ_ERR_SHAPE, "f32 GEMM: too many rows");
  MINQ_CUDA_TRY(launch_k(f32_gemm_kernel, dim3((unsigned)grid), dim3(kFgThreads), kFgSmem, s, w,
                         rows, cols, x, x_stride, B, y, y_stride));
  return MINQ_OK;
}

}  // namespace minq
