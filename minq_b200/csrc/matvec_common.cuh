// Shared pieces of the matvec kernels: parameters, x staging with the fused
// RMSNorm prologue (tensor.rs:219-227), exact code -> float conversion and
// the 8-column partial dot of one lane.
#pragma once

#include "common.cuh"

namespace minq {

struct MatvecParams {
  const uint8_t* w0;     // quantized [rows, nb blocks] (or f32 rows for the dense kernel)
  const uint8_t* w1;     // second matrix for the SwiGLU dual mode (up_proj), else null
  size_t rows;           // output rows
  int cols;              // input length
  const float* x;        // [cols]
  const float* norm_w;   // RMSNorm gain applied to x while staging, or null
  float eps;
  const float* bias;     // [rows] or null
  const float* residual; // [rows] or null: y = residual + W x (may alias y)
  float* y;              // [rows]
  int ks;                // warps per row group (column split, generic kernel)
  unsigned long long* argmax_part;  // per-CTA packed argmax (dense kernel), or null
  int* status;           // device status word (bounded-wait timeouts)
};

// xs (shared) = xs * (1/sqrt(mean(xs^2)+eps)) * w; w in global or shared
// memory. The sum of squares is a block reduction. Ends with __syncthreads().
__device__ __forceinline__ void block_rms_scale(const MatvecParams& p, float* xs, const float* w,
                                                float* red, bool vec) {
  const int tid = threadIdx.x, nt = blockDim.x;
  float ss = 0.0f;
  if (vec) {
    const float4* xs4 = reinterpret_cast<const float4*>(xs);
#pragma unroll 4
    for (int i = tid; i < (p.cols >> 2); i += nt) {
      const float4 v = xs4[i];
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
  } else {
    for (int i = tid; i < p.cols; i += nt) ss = fmaf(xs[i], xs[i], ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : 0.0f;
    v = warp_sum(v);
    if (tid == 0) red[32] = 1.0f / sqrtf(v / (float)p.cols + p.eps);
  }
  __syncthreads();
  const float inv = red[32];
  if (vec) {
    float4* xs4 = reinterpret_cast<float4*>(xs);
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll 4
    for (int i = tid; i < (p.cols >> 2); i += nt) {
      float4 v = xs4[i];
      const float4 g = w4[i];
      v.x = v.x * inv * g.x;
      v.y = v.y * inv * g.y;
      v.z = v.z * inv * g.z;
      v.w = v.w * inv * g.w;
      xs4[i] = v;
    }
  } else {
    for (int i = tid; i < p.cols; i += nt) xs[i] = xs[i] * inv * w[i];
  }
  __syncthreads();
}

// Stage x (optionally RMS-normalised) into shared memory with ordinary loads.
// `red` needs 33 floats. Ends with __syncthreads().
__device__ __forceinline__ void stage_x(const MatvecParams& p, float* xs, float* red) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool vec = (p.cols & 3) == 0 && ((uintptr_t)p.x & 15) == 0 &&
                   (!p.norm_w || ((uintptr_t)p.norm_w & 15) == 0);
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    float4* xs4 = reinterpret_cast<float4*>(xs);
#pragma unroll 4
    for (int i = tid; i < (p.cols >> 2); i += nt) xs4[i] = x4[i];
  } else {
    for (int i = tid; i < p.cols; i += nt) xs[i] = p.x[i];
  }
  __syncthreads();
  if (p.norm_w) block_rms_scale(p, xs, p.norm_w, red, vec);
}

// Byte k of w placed in the low mantissa byte of 2^23: value 2^23 + byte.
__device__ __forceinline__ float byte_to_float(uint32_t w, int k) {
  return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7440u | (unsigned)k));
}

__device__ __forceinline__ float2 bytes_to_float2(uint32_t w, int k0, int k1) {
  return make_float2(byte_to_float(w, k0), byte_to_float(w, k1));
}

// Partial dot of one lane's 8 columns of one block (scale not applied), from
// the lane's code word(s): Q8_0 two words (8 x i8), Q4_0 one word (8
// nibbles: byte i holds columns 2i (low) and 2i+1 (high), quantize.rs:8-10).
// Codes become exact floats (2^23 + code - magic), then packed f32x2 FMAs.
template <int DT>
__device__ __forceinline__ float dot8(uint32_t c0, uint32_t c1, const float4& xa,
                                      const float4& xb) {
  float2 a, b, s;
  if (DT == MINQ_Q8_0) {
    const uint32_t w0 = c0 ^ 0x80808080u;  // i8 -> u8 offset by 128
    const uint32_t w1 = c1 ^ 0x80808080u;
    const float2 k = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    a = __fadd2_rn(bytes_to_float2(w0, 0, 1), k);
    b = __fadd2_rn(bytes_to_float2(w0, 2, 3), k);
    s = __fmul2_rn(a, make_float2(xa.x, xa.y));
    s = __ffma2_rn(b, make_float2(xa.z, xa.w), s);
    a = __fadd2_rn(bytes_to_float2(w1, 0, 1), k);
    b = __fadd2_rn(bytes_to_float2(w1, 2, 3), k);
    s = __ffma2_rn(a, make_float2(xb.x, xb.y), s);
    s = __ffma2_rn(b, make_float2(xb.z, xb.w), s);
  } else {
    const uint32_t lo = c0 & 0x0F0F0F0Fu;         // columns 0,2,4,6
    const uint32_t hi = (c0 >> 4) & 0x0F0F0F0Fu;  // columns 1,3,5,7
    // interleave to column order: (0,1) (2,3) (4,5) (6,7)
    const uint32_t p01 = __byte_perm(lo, hi, 0x5140);  // lo0 hi0 lo1 hi1
    const uint32_t p23 = __byte_perm(lo, hi, 0x7362);  // lo2 hi2 lo3 hi3
    const float2 k = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    a = __fadd2_rn(bytes_to_float2(p01, 0, 1), k);
    b = __fadd2_rn(bytes_to_float2(p01, 2, 3), k);
    s = __fmul2_rn(a, make_float2(xa.x, xa.y));
    s = __ffma2_rn(b, make_float2(xa.z, xa.w), s);
    a = __fadd2_rn(bytes_to_float2(p23, 0, 1), k);
    b = __fadd2_rn(bytes_to_float2(p23, 2, 3), k);
    s = __ffma2_rn(a, make_float2(xb.x, xb.y), s);
    s = __ffma2_rn(b, make_float2(xb.z, xb.w), s);
  }
  return s.x + s.y;
}

// Lane partial dot with the block read from global memory (generic path).
template <int DT>
__device__ __forceinline__ float lane_dot(const uint8_t* blk, int sub, const float4& xa,
                                          const float4& xb) {
  if (DT == MINQ_Q8_0) {
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(blk + 4 + 8 * sub);
    return dot8<DT>(__ldg(wp), __ldg(wp + 1), xa, xb);
  }
  return dot8<DT>(__ldg(reinterpret_cast<const uint32_t*>(blk + 4 + 4 * sub)), 0u, xa, xb);
}

// Same with the block staged in shared memory.
template <int DT>
__device__ __forceinline__ float lane_dot_smem(const unsigned char* blk, int sub,
                                               const float4& xa, const float4& xb) {
  if (DT == MINQ_Q8_0) {
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(blk + 4 + 8 * sub);
    return dot8<DT>(wp[0], wp[1], xa, xb);
  }
  return dot8<DT>(*reinterpret_cast<const uint32_t*>(blk + 4 + 4 * sub), 0u, xa, xb);
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

}  // namespace minq
