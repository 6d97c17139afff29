// Small kernels of the forward step that are not fused into a matvec:
// embedding row gather (model.rs:275), standalone RMSNorm (tensor.rs:219-227,
// dense-f32 layers), bias/residual epilogue (tensor.rs:195 add_) and SwiGLU
// (tensor.rs:203-215) after f32 matvecs, the device-side position
// counter of a graph-captured decode step, and the per-position negative
// log-likelihood of perplexity evaluation (ppl.rs:30-35).
#include "common.cuh"

namespace minq {

__global__ void embed_kernel(const float* __restrict__ embed, const uint32_t* tok, size_t vocab,
                             int hidden, float* __restrict__ x) {
  pdl_wait();
  pdl_launch_dependents();
  uint32_t t = *tok;
  if (t >= vocab) t = 0;  // host validates tokens; never read out of bounds
  const float* row = embed + (size_t)t * hidden;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
    x[i] = row[i];
}

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float eps, int n, float* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[33];
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[32] = 1.0f / sqrtf(v / (float)n + eps);
  }
  __syncthreads();
  const float inv = red[32];
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = x[i] * inv * w[i];
}

__global__ void epilogue_kernel(const float* acc, const float* bias, const float* residual,
                                float* y, size_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float v = acc[i];
    if (bias) v += bias[i];
    if (residual) v = residual[i] + v;
    y[i] = v;
  }
}

__global__ void swiglu_kernel(const float* g, const float* u, float* h, size_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = g[i];
    h[i] = (v / (1.0f + expf(-v))) * u[i];
  }
}

__global__ void advance_pos_kernel(int* pos, int by) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) *pos += by;
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ppl.rs:30-35 for row blockIdx.x of logits [rows][V]: the f32 max (a fold
// with f32::max, NaN ignored; the order of a max does not matter), then
// sum_i exp((l_i - max) as f64) in f64, and nll = max + ln(sum) - l[target].
// The f64 sum is a tree instead of the reference's left-to-right fold (a
// relative difference of order 1e-16 per term). A target outside the row
// (the host checks the tokens first) gives NaN rather than a read.
__global__ void __launch_bounds__(1024) nll_rows_kernel(const float* __restrict__ logits, size_t V,
                                                        const uint32_t* __restrict__ targets,
                                                        double* __restrict__ out) {
  __shared__ float smx[32];
  __shared__ double ssum[32];
  pdl_wait();
  const float* row = logits + (size_t)blockIdx.x * V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  float mx = -INFINITY;
  for (size_t i = tid; i < V; i += blockDim.x) mx = fmaxf(mx, row[i]);
  mx = warp_max(mx);
  if (lane == 0) smx[warp] = mx;
  __syncthreads();
  mx = warp_max(lane < nw ? smx[lane] : -INFINITY);
  double sum = 0.0;
  for (size_t i = tid; i < V; i += blockDim.x) sum += exp((double)(row[i] - mx));
  sum = warp_sum_f64(sum);
  if (lane == 0) ssum[warp] = sum;
  __syncthreads();
  if (warp == 0) {
    sum = warp_sum_f64(lane < nw ? ssum[lane] : 0.0);
    if (lane == 0) {
      const uint32_t t = targets[blockIdx.x];
      out[blockIdx.x] = t < V ? (double)mx + log(sum) - (double)row[t] : (double)NAN;
    }
  }
  pdl_launch_dependents();
}

static unsigned ew_grid(size_t n) {
  size_t g = (n + 255) / 256;
  size_t cap = (size_t)sm_count() * 8;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

minq_status launch_embed(const float* embed, const uint32_t* d_tok, size_t vocab, int hidden,
                         float* x, cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(embed_kernel, dim3((hidden + 255) / 256), dim3(256), 0, s, embed, d_tok,
                         vocab, hidden, x));
  MINQ_LAUNCH_CHECK("embed_kernel");
  return MINQ_OK;
}

minq_status launch_rmsnorm(const float* x, const float* w, float eps, int n, float* out,
                           cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(rmsnorm_kernel, dim3(1), dim3(1024), 0, s, x, w, eps, n, out));
  MINQ_LAUNCH_CHECK("rmsnorm_kernel");
  return MINQ_OK;
}

minq_status launch_epilogue(const float* acc, const float* bias, const float* residual, float* y,
                            size_t n, cudaStream_t s) {
  MINQ_CUDA_TRY(
      launch_k(epilogue_kernel, dim3(ew_grid(n)), dim3(256), 0, s, acc, bias, residual, y, n));
  MINQ_LAUNCH_CHECK("epilogue_kernel");
  return MINQ_OK;
}

minq_status launch_swiglu(const float* g, const float* u, float* h, size_t n, cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(swiglu_kernel, dim3(ew_grid(n)), dim3(256), 0, s, g, u, h, n));
  MINQ_LAUNCH_CHECK("swiglu_kernel");
  return MINQ_OK;
}

minq_status launch_nll_rows(const float* logits, size_t V, int rows, const uint32_t* targets,
                            double* out, cudaStream_t s) {
  if (rows <= 0) return MINQ_OK;
  MINQ_CUDA_TRY(launch_k(nll_rows_kernel, dim3((unsigned)rows), dim3(1024), 0, s, logits, V,
                         targets, out));
  MINQ_LAUNCH_CHECK("nll_rows_kernel");
  return MINQ_OK;
}

minq_status launch_advance_pos(int* pos, int by, cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(advance_pos_kernel, dim3(1), dim3(32), 0, s, pos, by));
  MINQ_LAUNCH_CHECK("advance_pos_kernel");
  return MINQ_OK;
}

}  // namespace minq
