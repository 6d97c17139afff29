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
//
// The launch's bounded device-side waits report a timeout into a second
// file-scope word, g_attn_static_status, instead of the allocated status
// word of the other entry points; minq_attend_static_status reads and clears
// it (and minq_device_status folds it in), again without allocating.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace minq {

// 32 MiB: n_heads x ceil(len / 32) x (head_dim + 2) floats + 256 bytes must
// fit, e.g. 32 heads of 128 up to len 64 512, or 14 heads of 64 up to 290 496.
constexpr size_t kStaticAttnScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_attn_scratch[kStaticAttnScratchBytes];
static __device__ int g_attn_static_status;

constexpr int kMaxDevices = 64;

struct StaticSlots {
  void* scratch = nullptr;
  int* status = nullptr;
};
static StaticSlots g_slots[kMaxDevices];
static std::mutex g_slots_mu;

static minq_status current_device(int* dev) {
  MINQ_CUDA_TRY(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices)
    return fail(MINQ_ERR_CUDA, "device ordinal " + std::to_string(*dev) + " out of range");
  return MINQ_OK;
}

// Device addresses of g_attn_scratch and g_attn_static_status on the
// current device (set up once per device).
static minq_status static_slots(StaticSlots* out) {
  int dev = -1;
  MINQ_TRY(current_device(&dev));
  std::lock_guard<std::mutex> g(g_slots_mu);
  StaticSlots& s = g_slots[dev];
  if (!s.scratch) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(g_attn_scratch)");
    void* w = nullptr;
    e = cudaGetSymbolAddress(&w, g_attn_static_status);
    if (e != cudaSuccess || !w) return cuda_fail(e, "cudaGetSymbolAddress(g_attn_static_status)");
    s.status = (int*)w;
    s.scratch = p;
  }
  *out = s;
  return MINQ_OK;
}

// Reads and clears this device's g_attn_static_status (a no-op on a device
// where minq_attend_static never ran). The caller has synchronised.
minq_status take_static_attn_status() {
  int dev = -1;
  MINQ_TRY(current_device(&dev));
  {
    std::lock_guard<std::mutex> g(g_slots_mu);
    if (!g_slots[dev].status) return MINQ_OK;
  }
  int v = 0;
  MINQ_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_attn_static_status, sizeof(int)));
  if (v == 0) return MINQ_OK;
  const int zero = 0;
  MINQ_CUDA_TRY(cudaMemcpyToSymbol(g_attn_static_status, &zero, sizeof(int)));
  return fail(MINQ_ERR_TIMEOUT, "a bounded device-side wait in minq_attend_static timed out (status " +
                                    std::to_string(v) + ")");
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
  if (head_dim > 256)
    return fail(MINQ_ERR_SHAPE, "unsupported head_dim " + std::to_string(head_dim) +
                                    " (supported: 8, 16, 32, 64, 128, 256)");
  if (n_heads > 4096 || len > (size_t)INT32_MAX)
    return fail(MINQ_ERR_SHAPE, "n_heads must be <= 4096 and len <= 2^31 - 1");
  // Largest scratch any split choice of the attention launch can use.
  const size_t need = (size_t)n_heads * ((len + 31) / 32) * (head_dim + 2) * sizeof(float) + 256;
  if (need > kStaticAttnScratchBytes)
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
  StaticSlots slots;
  MINQ_TRY(static_slots(&slots));
  return launch_attention(q, k, v, 1, (int)n_heads, (int)n_kv, (int)head_dim, (int)len, 0,
                          head_dim, kvd, out, slots.scratch, kStaticAttnScratchBytes,
                          (cudaStream_t)stream, nullptr, 0, /*record_status=*/true,
                          /*len_step=*/0, slots.status);
}

extern "C" minq_status minq_attend_static_status(void) {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(MINQ_ERR_CUDA, "no CUDA device available (the CUDA path has no CPU fallback)");
  MINQ_CUDA_TRY(cudaDeviceSynchronize());
  return take_static_attn_status();
}
