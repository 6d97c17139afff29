// Shared device/host helpers for the minq B200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/minq_cuda.h"

namespace minq {

constexpr int kBlock = 32;     // quantize.rs:23 BLOCK_SIZE
constexpr int kQ8Bytes = 36;   // quantize.rs:25
constexpr int kQ4Bytes = 20;   // quantize.rs:27

inline int block_bytes(int dtype) { return dtype == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes; }

// Thread-local error text behind minq_last_error().
void set_error(const std::string& msg);
minq_status fail(minq_status code, const std::string& msg);
minq_status cuda_fail(cudaError_t e, const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Raise a kernel's dynamic shared-memory limit to at least `bytes` when its
// static plus `bytes` of dynamic shared memory exceed the 48 KB default
// (cached per device and kernel, so the attribute call happens once).
minq_status ensure_dynamic_smem(const void* kernel, size_t bytes);

// Per-device status word that bounded device-side waits set on timeout
// (allocated once per device), and its synchronous read-and-clear.
int* device_status_word();
minq_status take_device_status();
// Read-and-clear of minq_attend_static's file-scope status word on the
// current device (no allocation; the caller has synchronised).
minq_status take_static_attn_status();

#define MINQ_CUDA_TRY(expr)                                    \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::minq::cuda_fail(_e, #expr); \
  } while (0)

#define MINQ_TRY(expr)                     \
  do {                                     \
    minq_status _s = (expr);               \
    if (_s != MINQ_OK) return _s;          \
  } while (0)

// Launch counter behind minq_kernel_launches(): launch_k counts every launch
// it makes; the few launches made without it count themselves.
void count_launch();

// Check the last launch error.
#define MINQ_LAUNCH_CHECK(what)                                     \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return ::minq::cuda_fail(_e, what);      \
  } while (0)

// Programmatic dependent launch (PDL): every kernel of this library calls
// pdl_wait() before it reads or writes anything a preceding kernel on the
// stream touches, so any launch may carry the programmatic-serialization
// attribute; work that depends on nothing (weight prefetch) goes before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launches carry the PDL attribute (MINQ_PDL=0 disables it).
bool pdl_enabled();

// Every kernel of the library asks for the largest shared-memory carveout
// (cached per device and kernel), so an SM never has to drain to change its
// L1/shared split between two kernels of a stream: the next kernel's CTAs can
// become resident beside the running ones (Programmatic Dependent Launch).
void prefer_max_shared(const void* kernel);

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, Args&&... args) {
  prefer_max_shared(reinterpret_cast<const void*>(kernel));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Key that orders floats like Rust's f32::total_cmp (sampler.rs:10-17):
// -NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN.
__device__ __host__ __forceinline__ int32_t total_key(float f) {
#ifdef __CUDA_ARCH__
  int32_t b = __float_as_int(f);
#else
  int32_t b;
  memcpy(&b, &f, 4);
#endif
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// Pack (key, index) so that a larger packed value wins and ties go to the
// lower index: high 32 bits = order-preserving unsigned key, low 32 bits =
// ~index.
__device__ __forceinline__ unsigned long long argmax_pack(float v, uint32_t idx) {
  uint32_t ukey = (uint32_t)total_key(v) ^ 0x80000000u;
  return ((unsigned long long)ukey << 32) | (unsigned long long)(~idx);
}

__device__ __forceinline__ uint32_t argmax_unpack_index(unsigned long long p) {
  return ~(uint32_t)(p & 0xffffffffull);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

}  // namespace minq
