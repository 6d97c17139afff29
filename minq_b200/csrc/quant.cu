// GPU block quantizer / dequantizer, bit-identical to quantize.rs:78-166.
//
// One warp per 32-value block: lane i owns value i. The block amax is a warp
// max of fmaxf(0, |v|) — max is exact and order-independent, and starting
// from 0 reproduces the reference's `fold(0.0, f32::max)` including its
// NaN-skipping. d = amax / {127, 8} and id = 1 / d are IEEE-correct divisions
// (the library is built without fast-math), `roundf` rounds half away from
// zero like Rust's `f32::round`, and a NaN product casts to code 0 like
// Rust's saturating `as` cast.
#include "common.cuh"

namespace minq {

__device__ __forceinline__ int clamp_cast(float v, float lo, float hi) {
  if (isnan(v)) return 0;
  float c = v < lo ? lo : (v > hi ? hi : v);
  return (int)c;
}

template <int DT>
__global__ void quantize_kernel(const float* __restrict__ x, size_t nblocks,
                                uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t b = warp; b < nblocks; b += nwarps) {
    float v = x[b * kBlock + lane];
    float a = warp_max(fmaxf(0.0f, fabsf(v)));
    if (DT == MINQ_Q8_0) {
      uint8_t* o = out + b * kQ8Bytes;
      float d = a / 127.0f;
      int q = 0;
      if (d != 0.0f) {
        float id = 1.0f / d;
        q = clamp_cast(roundf(__fmul_rn(v, id)), -127.0f, 127.0f);
      }
      if (lane == 0) {
        uint32_t bits = __float_as_uint(d);
        o[0] = bits & 0xff;
        o[1] = (bits >> 8) & 0xff;
        o[2] = (bits >> 16) & 0xff;
        o[3] = bits >> 24;
      }
      o[4 + lane] = (uint8_t)(int8_t)q;
    } else {
      uint8_t* o = out + b * kQ4Bytes;
      float d = a / 8.0f;
      uint32_t code = 0;  // d == 0 packs 0x00 bytes, not 0x88 (quantize.rs:127-139)
      if (d != 0.0f) {
        float id = 1.0f / d;
        code = (uint32_t)(clamp_cast(roundf(__fmul_rn(v, id)), -8.0f, 7.0f) + 8);
      }
      uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
      if (lane == 0) {
        uint32_t bits = __float_as_uint(d);
        o[0] = bits & 0xff;
        o[1] = (bits >> 8) & 0xff;
        o[2] = (bits >> 16) & 0xff;
        o[3] = bits >> 24;
      }
      if ((lane & 1) == 0) o[4 + lane / 2] = (uint8_t)(code | (hi << 4));
    }
  }
}

template <int DT>
__global__ void dequantize_kernel(const uint8_t* __restrict__ in, size_t nblocks,
                                  float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t b = warp; b < nblocks; b += nwarps) {
    if (DT == MINQ_Q8_0) {
      const uint8_t* blk = in + b * kQ8Bytes;
      uint32_t bits = blk[0] | (blk[1] << 8) | (blk[2] << 16) | ((uint32_t)blk[3] << 24);
      float d = __uint_as_float(bits);
      out[b * kBlock + lane] = __fmul_rn((float)(int8_t)blk[4 + lane], d);
    } else {
      const uint8_t* blk = in + b * kQ4Bytes;
      uint32_t bits = blk[0] | (blk[1] << 8) | (blk[2] << 16) | ((uint32_t)blk[3] << 24);
      float d = __uint_as_float(bits);
      uint8_t byte = blk[4 + lane / 2];
      int c = (lane & 1) ? (byte >> 4) : (byte & 0x0F);
      out[b * kBlock + lane] = __fmul_rn((float)(c - 8), d);
    }
  }
}

static unsigned grid_for_warps(size_t nwarps) {
  size_t g = (nwarps + 7) / 8;  // 8 warps per 256-thread CTA
  size_t cap = (size_t)sm_count() * 64;
  if (g > cap) g = cap;
  if (g == 0) g = 1;
  return (unsigned)g;
}

minq_status launch_quantize(int dtype, const float* x, size_t n, void* out, cudaStream_t s) {
  size_t nb = n / kBlock;
  if (nb == 0) return MINQ_OK;
  unsigned grid = grid_for_warps(nb);
  if (dtype == MINQ_Q8_0)
    quantize_kernel<MINQ_Q8_0><<<grid, 256, 0, s>>>(x, nb, (uint8_t*)out);
  else
    quantize_kernel<MINQ_Q4_0><<<grid, 256, 0, s>>>(x, nb, (uint8_t*)out);
  count_launch();
  MINQ_LAUNCH_CHECK("quantize_kernel");
  return MINQ_OK;
}

minq_status launch_dequantize(int dtype, const void* in, size_t nblocks, float* out,
                              cudaStream_t s) {
  if (nblocks == 0) return MINQ_OK;
  unsigned grid = grid_for_warps(nblocks);
  if (dtype == MINQ_Q8_0)
    dequantize_kernel<MINQ_Q8_0><<<grid, 256, 0, s>>>((const uint8_t*)in, nblocks, out);
  else
    dequantize_kernel<MINQ_Q4_0><<<grid, 256, 0, s>>>((const uint8_t*)in, nblocks, out);
  count_launch();
  MINQ_LAUNCH_CHECK("dequantize_kernel");
  return MINQ_OK;
}

}  // namespace minq
