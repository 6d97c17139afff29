// minq_attend_static: the attention of minq_attend (model.rs:223-248) with
// its split-KV scratch in a file-scope device array instead of a caller
// workspace, so the call allocates no device memory at all (no cudaMalloc,
// no cudaFree, no allocating library routine).
//
// The scratch holds the per-split partial outputs and (max, sum) pairs of
// the split-KV pass; every split writes its own partials before the combine
// kernel reads them, so nothing in it has to start at zero. Its address is
// taken once per device with cudaGetSymbolAddress, under that device, the
// first time the entry point runs there.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace minq {

// 32 MiB: n_heads x ceil(len / 32) x (head_dim + 2) floats + 256 bytes must
// fit, e.g. 32 heads of 128 up to len 64 512, or 14 heads of 64 up to 290 496.
constexpr size_t kStaticAttnScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_attn_scratch[kStaticAttnScratchBytes];

constexpr int kMaxDevices = 64;

// Device address of g_attn_scratch on the current device (set up once).
static minq_status static_scratch(void** out) {
  static void* ptrs[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = -1;
  MINQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MINQ_ERR_CUDA, "device ordinal " + std::to_string(dev) + " out of range");
  std::lock_guard<std::mutex> g(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(g_attn_scratch)");
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return MINQ_OK;
}

}  // namespace minq

using namespace minq;

extern "C" minq_status minq_attend_static(const float* q, const float* k, const float* v,
                                          size_t len, size_t n_heads, size_t n_kv,
                                          size_t head_dim, float* out, void* stream) {
  if (!q || !k || !v || !out) return fail(MINQ_ERR_ARG, "null pointer");
  if (n_kv == 0 || n_heads % n_kv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  if (len == 0) return fail(MINQ_ERR_SHAPE, "attention over an empty history");
  // Largest scratch any split choice of the attention launch can use.
  const size_t need = (size_t)n_heads * ((len + 31) / 32) * (head_dim + 2) * sizeof(float) + 256;
  if (len > (size_t)INT32_MAX || n_heads > 4096 || head_dim > 256 ||
      need > kStaticAttnScratchBytes)
    return fail(MINQ_ERR_ARG,
                "minq_attend_static: n_heads x ceil(len/32) x (head_dim+2) x 4 + 256 = " +
                    std::to_string(need) + " bytes exceeds its static scratch of " +
                    std::to_string(kStaticAttnScratchBytes) +
                    " bytes; use minq_attend with a workspace");
  const size_t kvd = n_kv * head_dim;
  if (head_dim >= 16 && (kvd % 4 != 0 || (uintptr_t)k % 16 != 0 || (uintptr_t)v % 16 != 0))
    return fail(MINQ_ERR_ARG, "k/v must be 16-byte aligned");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(MINQ_ERR_CUDA, "no CUDA device available (the CUDA path has no CPU fallback)");
  void* scratch = nullptr;
  MINQ_TRY(static_scratch(&scratch));
  return launch_attention(q, k, v, 1, (int)n_heads, (int)n_kv, (int)head_dim, (int)len, 0,
                          head_dim, kvd, out, scratch, kStaticAttnScratchBytes,
                          (cudaStream_t)stream, nullptr, 0, /*record_status=*/false);
}
