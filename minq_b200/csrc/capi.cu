// Op-level C ABI entry points (include/minq_cuda.h) and error plumbing.
#include <atomic>
#include <cstdlib>
#include <map>
#include <set>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "ktimer.h"

namespace minq {

static thread_local std::string g_error;
static std::atomic<uint64_t> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_error = msg; }

minq_status fail(minq_status code, const std::string& msg) {
  g_error = msg;
  return code;
}

minq_status cuda_fail(cudaError_t e, const char* what) {
  g_error = std::string("cuda error in ") + what + ": " + cudaGetErrorString(e);
  return MINQ_ERR_CUDA;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MINQ_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

minq_status ensure_dynamic_smem(const void* kernel, size_t bytes) {
  if (bytes == 0) return MINQ_OK;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  size_t& cur = done[{dev, kernel}];
  if (cur >= bytes) return MINQ_OK;
  // without the opt-in, static + dynamic shared memory must stay within
  // 48 KB, so the kernel's static arrays count against that default
  cudaFuncAttributes fa{};
  MINQ_CUDA_TRY(cudaFuncGetAttributes(&fa, kernel));
  if (fa.sharedSizeBytes + bytes <= 48 * 1024) {
    cur = bytes;
    return MINQ_OK;
  }
  MINQ_CUDA_TRY(
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  cur = bytes;
  return MINQ_OK;
}

void prefer_max_shared(const void* kernel) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  if (done.insert({dev, kernel}).second)
    cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                         (int)cudaSharedmemCarveoutMaxShared);
}

int* device_status_word() {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (!words[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    words[dev] = p;
  }
  return words[dev];
}

minq_status take_device_status() {
  int* w = device_status_word();
  if (!w) return MINQ_OK;
  int v = 0;
  MINQ_CUDA_TRY(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (v == 0) return MINQ_OK;
  MINQ_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
  return fail(MINQ_ERR_TIMEOUT,
              "a bounded device-side wait timed out (status " + std::to_string(v) + ")");
}

static minq_status require_device() {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(MINQ_ERR_CUDA, "no CUDA device available (the CUDA path has no CPU fallback)");
  return MINQ_OK;
}

static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

// ---- kernel timer ----
namespace {
struct TimerState {
  std::mutex mu;
  KFamily fam = KF_NONE;
  std::vector<cudaEvent_t> pool;  // pairs: [2i] start, [2i+1] stop
  size_t used = 0;
  double bytes = 0.0;
};
TimerState& timer() {
  static TimerState t;
  return t;
}
}  // namespace

bool timer_active(KFamily fam) { return fam != KF_NONE && timer().fam == fam; }

static cudaEvent_t timer_event() {
  TimerState& t = timer();
  if (t.used == t.pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    t.pool.push_back(e);
  }
  return t.pool[t.used++];
}

void timer_before(cudaStream_t s) {
  std::lock_guard<std::mutex> g(timer().mu);
  cudaEventRecord(timer_event(), s);
}

void timer_after(cudaStream_t s, double bytes) {
  std::lock_guard<std::mutex> g(timer().mu);
  cudaEventRecord(timer_event(), s);
  timer().bytes += bytes;
}

}  // namespace minq

using namespace minq;

extern "C" {

const char* minq_last_error(void) { return g_error.c_str(); }

int minq_abi_version(void) { return MINQ_ABI_VERSION; }

uint64_t minq_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

minq_status minq_device_status(void) {
  MINQ_TRY(require_device());
  MINQ_CUDA_TRY(cudaDeviceSynchronize());
  const minq_status a = take_device_status();
  const minq_status b = take_static_attn_status();
  return a != MINQ_OK ? a : b;
}

minq_status minq_kernel_timer_start(const char* family) {
  if (!family) return fail(MINQ_ERR_ARG, "null family");
  std::string f(family);
  KFamily fam = f == "qmatvec" ? KF_QMATVEC
                : f == "f32_matvec" ? KF_F32_MATVEC
                : f == "attention" ? KF_ATTENTION : KF_NONE;
  if (fam == KF_NONE) return fail(MINQ_ERR_ARG, "unknown kernel family `" + f + "`");
  TimerState& t = timer();
  std::lock_guard<std::mutex> g(t.mu);
  t.fam = fam;
  t.used = 0;
  t.bytes = 0.0;
  return MINQ_OK;
}

minq_status minq_kernel_timer_stop(uint64_t* launches, double* total_ms, double* bytes) {
  TimerState& t = timer();
  std::lock_guard<std::mutex> g(t.mu);
  t.fam = KF_NONE;
  double ms = 0.0;
  for (size_t i = 0; i + 1 < t.used; i += 2) {
    MINQ_CUDA_TRY(cudaEventSynchronize(t.pool[i + 1]));
    float e = 0.0f;
    MINQ_CUDA_TRY(cudaEventElapsedTime(&e, t.pool[i], t.pool[i + 1]));
    ms += e;
  }
  if (launches) *launches = t.used / 2;
  if (total_ms) *total_ms = ms;
  if (bytes) *bytes = t.bytes;
  t.used = 0;
  t.bytes = 0.0;
  return MINQ_OK;
}

minq_status minq_quantize(minq_dtype dtype, const float* x, size_t n, void* out, void* stream) {
  if (dtype != MINQ_Q8_0 && dtype != MINQ_Q4_0) return fail(MINQ_ERR_FORMAT, "unknown dtype");
  if (n % kBlock != 0)
    return fail(MINQ_ERR_SHAPE, "quantization requires a multiple of 32 elements, got " +
                                    std::to_string(n));
  if (n && (!x || !out)) return fail(MINQ_ERR_ARG, "null pointer");
  MINQ_TRY(require_device());
  return launch_quantize(dtype, x, n, out, (cudaStream_t)stream);
}

minq_status minq_dequantize(minq_dtype dtype, const void* blocks, size_t nbytes, float* out,
                            size_t n_out, void* stream) {
  if (dtype != MINQ_Q8_0 && dtype != MINQ_Q4_0) return fail(MINQ_ERR_FORMAT, "unknown dtype");
  const size_t bb = block_bytes(dtype);
  if (nbytes % bb != 0 || n_out != nbytes / bb * kBlock)
    return fail(MINQ_ERR_SHAPE, std::string("dequantize_") + (dtype == MINQ_Q8_0 ? "q8_0" : "q4_0") +
                                    ": " + std::to_string(nbytes) + " bytes vs " +
                                    std::to_string(n_out) + " outputs");
  if (nbytes && (!blocks || !out)) return fail(MINQ_ERR_ARG, "null pointer");
  MINQ_TRY(require_device());
  return launch_dequantize(dtype, blocks, nbytes / bb, out, (cudaStream_t)stream);
}

minq_status minq_qmatvec(minq_dtype dtype, const void* blocks, size_t rows, size_t cols,
                         const float* x, size_t x_len, float* y, void* stream) {
  if (dtype != MINQ_Q8_0 && dtype != MINQ_Q4_0) return fail(MINQ_ERR_FORMAT, "unknown dtype");
  if (x_len != cols)
    return fail(MINQ_ERR_SHAPE, "quantized matvec: " + std::to_string(cols) +
                                    " cols vs input len " + std::to_string(x_len));
  if (cols % kBlock != 0) return fail(MINQ_ERR_SHAPE, "cols must be a multiple of 32");
  if (cols > (1u << 30)) return fail(MINQ_ERR_SHAPE, "cols too large");
  if (rows == 0) return MINQ_OK;
  if (!blocks || !x || !y) return fail(MINQ_ERR_ARG, "null pointer");
  if (!aligned(blocks, 4) || !aligned(x, 16))
    return fail(MINQ_ERR_ARG, "blocks must be 4-byte and x 16-byte aligned");
  MINQ_TRY(require_device());
  return launch_qmatvec(dtype, blocks, nullptr, rows, (int)cols, x, nullptr, 0.0f, nullptr,
                        nullptr, y, (cudaStream_t)stream);
}

size_t minq_qmatmul_workspace_bytes(size_t batch, size_t rows, size_t cols) {
  // prepared inputs (x_hi + x_lo: batch x cols floats) and up to 16 column
  // slices of partial sums (16 x batch x rows floats)
  return 4 * batch * cols + 64 * batch * rows + 256;
}

minq_status minq_qmatmul(minq_dtype dtype, const void* blocks, size_t rows, size_t cols,
                         const float* x, size_t batch, float* y, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (dtype != MINQ_Q8_0 && dtype != MINQ_Q4_0) return fail(MINQ_ERR_FORMAT, "unknown dtype");
  if (cols % kBlock != 0) return fail(MINQ_ERR_SHAPE, "cols must be a multiple of 32");
  if (cols > (1u << 30) || rows > (1u << 30)) return fail(MINQ_ERR_SHAPE, "matrix too large");
  if (batch < 1 || batch > (size_t)kQmmMaxB) return fail(MINQ_ERR_ARG, "batch must be 1..64");
  if (rows == 0) return MINQ_OK;
  if (!blocks || !x || !y || !workspace) return fail(MINQ_ERR_ARG, "null pointer");
  if (!aligned(blocks, 16) || !aligned(x, 16) || !aligned(workspace, 16))
    return fail(MINQ_ERR_ARG, "blocks, x and workspace must be 16-byte aligned");
  if (workspace_bytes < minq_qmatmul_workspace_bytes(batch, rows, cols))
    return fail(MINQ_ERR_ARG, "workspace smaller than minq_qmatmul_workspace_bytes");
  MINQ_TRY(require_device());
  float* xp = static_cast<float*>(workspace);
  const size_t xp_floats = batch * cols;
  float* part = xp + xp_floats;
  const size_t part_floats = 16 * batch * rows;
  return launch_qmatmul(dtype, blocks, nullptr, rows, (int)cols, (int)batch, x, cols, nullptr,
                        0.0f, xp, xp_floats, nullptr, nullptr, y, rows, part, part_floats,
                        (cudaStream_t)stream);
}

minq_status minq_matvec_f32(const float* w, size_t rows, size_t cols, const float* x,
                            size_t x_len, float* y, void* stream) {
  if (x_len != cols)
    return fail(MINQ_ERR_SHAPE, "matvec: weight cols " + std::to_string(cols) +
                                    " vs input len " + std::to_string(x_len));
  if (cols % 4 != 0) return fail(MINQ_ERR_SHAPE, "f32 matvec needs cols % 4 == 0");
  if (rows == 0) return MINQ_OK;
  if (!w || !x || !y) return fail(MINQ_ERR_ARG, "null pointer");
  if (!aligned(w, 16) || !aligned(x, 16)) return fail(MINQ_ERR_ARG, "w and x must be 16-byte aligned");
  MINQ_TRY(require_device());
  return launch_f32_matvec(w, rows, (int)cols, x, nullptr, 0.0f, y, nullptr, nullptr,
                           (cudaStream_t)stream);
}

minq_status minq_argmax(const float* logits, size_t n, uint32_t* out, void* stream) {
  if (!logits || !out) return fail(MINQ_ERR_ARG, "null pointer");
  MINQ_TRY(require_device());
  // Partials live in a small per-thread device buffer reused across calls.
  static thread_local unsigned long long* part = nullptr;
  static thread_local int part_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int cap = argmax_parts_capacity();
  if (!part || part_dev != dev) {
    MINQ_CUDA_TRY(cudaMalloc(&part, cap * sizeof(unsigned long long)));
    part_dev = dev;
  }
  if (n == 0) {
    MINQ_CUDA_TRY(cudaMemsetAsync(out, 0, 4, (cudaStream_t)stream));  // sampler.rs:16
    return MINQ_OK;
  }
  return launch_argmax(logits, n, part, cap, out, (cudaStream_t)stream);
}

size_t minq_attn_workspace_bytes(size_t batch, size_t n_heads, size_t max_len) {
  // split partials + the rotated queries of minq_attn_decode
  return attn_workspace_bytes(batch, n_heads, max_len, 256) + batch * n_heads * 256 * 4 + 512;
}

minq_status minq_attn_decode(const float* q, const float* k_new, const float* v_new,
                             const float* q_norm, const float* k_norm, float eps,
                             const float* rope_cos, const float* rope_sin, size_t batch,
                             size_t n_heads, size_t n_kv, size_t head_dim, size_t pos,
                             float* k_cache, float* v_cache, size_t seq_stride,
                             size_t head_stride, size_t pos_stride, float* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!q || !k_new || !v_new || !rope_cos || !rope_sin || !k_cache || !v_cache || !out)
    return fail(MINQ_ERR_ARG, "null pointer");
  if (batch == 0) return MINQ_OK;
  if (n_kv == 0 || n_heads % n_kv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  if (head_dim % 2 != 0) return fail(MINQ_ERR_MODEL, "head_dim must be even (RoPE)");
  if (head_dim >= 16 && ((seq_stride | head_stride | pos_stride) % 4 != 0 ||
                         !aligned(k_cache, 16) || !aligned(v_cache, 16)))
    return fail(MINQ_ERR_ARG, "cache strides must be multiples of 4 and bases 16-byte aligned");
  MINQ_TRY(require_device());
  cudaStream_t s = (cudaStream_t)stream;
  // The rotated queries live in the workspace tail, after the split partials.
  const size_t qbytes = batch * n_heads * head_dim * sizeof(float);
  const size_t need_attn = attn_workspace_bytes(batch, n_heads, pos + 1, head_dim);
  if (!workspace || workspace_bytes < need_attn + qbytes + 256)
    return fail(MINQ_ERR_ARG, "workspace too small: need " +
                                  std::to_string(need_attn + qbytes + 256) + " bytes");
  float* q_rot = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(workspace) + need_attn + 255) / 256 * 256);
  MINQ_TRY(launch_rope_append(q, k_new, v_new, n_heads * head_dim, n_kv * head_dim, q_norm,
                              k_norm, eps, rope_cos, rope_sin, batch, (int)n_heads, (int)n_kv,
                              (int)head_dim, (int)pos, q_rot, k_cache, v_cache, seq_stride,
                              head_stride, pos_stride, s));
  return launch_attention(q_rot, k_cache, v_cache, batch, (int)n_heads, (int)n_kv,
                          (int)head_dim, (int)pos + 1, seq_stride, head_stride, pos_stride, out,
                          workspace, need_attn, s);
}

minq_status minq_attend(const float* q, const float* k, const float* v, size_t len,
                        size_t n_heads, size_t n_kv, size_t head_dim, float* out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out) return fail(MINQ_ERR_ARG, "null pointer");
  if (n_kv == 0 || n_heads % n_kv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  const size_t kvd = n_kv * head_dim;
  if (head_dim >= 16 && (kvd % 4 != 0 || !aligned(k, 16) || !aligned(v, 16)))
    return fail(MINQ_ERR_ARG, "k/v must be 16-byte aligned");
  MINQ_TRY(require_device());
  return launch_attention(q, k, v, 1, (int)n_heads, (int)n_kv, (int)head_dim, (int)len, 0,
                          head_dim, kvd, out, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t minq_attn_prefill_workspace_bytes(size_t n_tokens, size_t n_heads, size_t n_kv,
                                         size_t head_dim) {
  if (n_tokens == 0 || n_tokens > (1u << 20) || n_heads > 4096 || head_dim > 256) return 0;
  return prefill_attention_workspace((int)n_tokens, (int)n_heads, (int)n_kv, (int)head_dim);
}

minq_status minq_attend_prefill(const float* q, const float* k_cache, const float* v_cache,
                                size_t head_stride, size_t p0, size_t n_tokens, size_t n_heads,
                                size_t n_kv, size_t head_dim, float* out, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(MINQ_ERR_ARG, "null pointer");
  if (n_kv == 0 || n_heads % n_kv != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  if (n_tokens == 0 || n_tokens > (1u << 20) || p0 > (1u << 30) || n_heads > 4096)
    return fail(MINQ_ERR_SHAPE, "prefill attention: token count or position out of range");
  if (!prefill_attention_supported((int)n_heads, (int)n_kv, (int)head_dim))
    return fail(MINQ_ERR_SHAPE, "unsupported head_dim " + std::to_string(head_dim) +
                                    " for prefill attention (supported: 64, 128)");
  MINQ_TRY(require_device());
  return launch_prefill_attention(q, k_cache, v_cache, head_stride, (int)p0, (int)n_tokens,
                                  (int)n_heads, (int)n_kv, (int)head_dim, out, workspace,
                                  workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
