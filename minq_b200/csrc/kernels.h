// Host launchers of the CUDA kernels (one declaration per .cu entry).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "../../include/minq_cuda.h"

namespace minq {

// tp_allreduce.cu: one-shot all-reduce of the residual stream over the
// tensor-parallel ranks through NVLink peer memory (receive buffers mapped
// by CUDA IPC; see the file's header comment).
struct TpAr {
  bool on = false;
  int world = 1, rank = 0, sites = 0, H = 0, ncta = 0;
  char* base = nullptr;                 // this rank's buffer (receive slots, then flags)
  float* recv = nullptr;                // [sites][world][H]
  int* flag = nullptr;                  // [sites][world][ncta]
  float** peer_recv = nullptr;          // device array [world]: every rank's receive slots
  int** peer_flag = nullptr;            // device array [world]: every rank's flags
  unsigned long long* step = nullptr;   // device token counter (the epoch)
  unsigned long long* ctr = nullptr;    // the decode megakernel's exchange epoch (low word)
  std::vector<void*> opened;            // IPC mappings of other processes' buffers
};
// Whether the peer path is wanted (MINQ_TP_NCCL=1 keeps the NCCL all-reduce).
bool tp_ar_wanted();
// Collective over the ranks of `nccl_comm`: allocate and map the buffers;
// ar->on stays false (the NCCL path) when any rank cannot map its peers.
minq_status tp_ar_setup(TpAr* ar, int rank, int world, int H, int sites, void* nccl_comm,
                        cudaStream_t s);
void tp_ar_release(TpAr* ar);
// x = sum over the ranks of x, all-reduce number `site` of the token.
minq_status launch_tp_allreduce(const TpAr& ar, float* x, int site, cudaStream_t s);
// The token's all-reduces are done: advance the epoch.
minq_status launch_tp_ar_advance(const TpAr& ar, cudaStream_t s);

// quant.cu
minq_status launch_quantize(int dtype, const float* x, size_t n, void* out, cudaStream_t s);
minq_status launch_dequantize(int dtype, const void* in, size_t nblocks, float* out,
                              cudaStream_t s);

// matvec.cu
// Launch plan of the TMA-fed quantized matvec (qmatvec_tma.cu).
struct QmvPlan {
  int nr;        // rows (row pairs in the dual mode) per CTA
  int stages;    // ring depth
  int nchunks;   // column chunks of 128
  size_t nctas;  // grid size
  size_t smem;   // dynamic shared memory bytes
};
QmvPlan plan_qmatvec_tma(int dtype, bool dual, size_t rows, int cols, bool norm);
bool qmatvec_uses_tma(int cols, const void* w0, const void* w1, const float* x,
                      const float* norm_w);
minq_status encode_qmatvec_map(const void* w, size_t rows, int cols, int dtype, int nr,
                               CUtensorMap* out);
// m0 / m1: optional tensor maps pre-encoded with plan_qmatvec_tma's nr.
minq_status launch_qmatvec(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                           const float* x, const float* norm_w, float eps, const float* bias,
                           const float* residual, float* y, cudaStream_t s,
                           const CUtensorMap* m0 = nullptr, const CUtensorMap* m1 = nullptr);
minq_status launch_f32_matvec(const float* w, size_t rows, int cols, const float* x,
                              const float* norm_w, float eps, float* y,
                              unsigned long long* argmax_part, int* n_part, cudaStream_t s);
minq_status launch_argmax_final(const unsigned long long* part, int n, uint32_t* out,
                                cudaStream_t s);
minq_status launch_argmax(const float* x, size_t n, unsigned long long* part, int n_part,
                          uint32_t* out, cudaStream_t s);
int argmax_parts_capacity();

// qmatmul.cu: Y[b] = W X[b] for up to kQmmMaxB inputs (see qmatmul.cu);
// w1 (dual) = up rows with a SwiGLU epilogue, else bias / residual; norm_w
// applies the input RMSNorm first; xn_scratch (xn_floats floats, at least
// B x cols) holds the prepared inputs; part (up to part_floats) holds the
// column slices' partials. From kQmmTcMinB quantized inputs on, the product
// runs on the tensor cores (qmatmul_tc.cu; measured on the LLaMA-3-8B
// shape: 3.3x faster than the CUDA-core kernel already at 8 inputs, 2.9x at
// 4), so the CUDA-core kernel serves one input and f32 weights below
// kF32GemmMinB inputs (from there on, f32_gemm.cu).
constexpr int kQmmMaxB = 64;
constexpr int kQmmTcMinB = 2;
minq_status launch_qmatmul(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                           int B, const float* x, size_t x_stride, const float* norm_w, float eps,
                           float* xn_scratch, size_t xn_floats, const float* bias,
                           const float* residual, float* y, size_t y_stride, float* part,
                           size_t part_floats, cudaStream_t s);
// f32_gemm.cu: Y[b] = W X[b] for dense f32 weights and kF32GemmMinB..64
// inputs (the tied lm_head over a perplexity chunk's positions or a batch),
// register-tiled on the CUDA cores; launch_qmatmul routes f32 weights
// without bias / residual there.
constexpr int kF32GemmMinB = 32;
bool f32_gemm_takes(int B, int cols, const void* w, const float* x, size_t x_stride);
minq_status launch_f32_gemm(const float* w, size_t rows, int cols, const float* x, size_t x_stride,
                            int B, float* y, size_t y_stride, cudaStream_t s);
// qmatmul_tc.cu: whether the tensor-core form takes the shape, and the launch.
bool qmatmul_tc_takes(int dtype, int cols, int B, size_t xp_floats);
minq_status launch_qmatmul_tc(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                              int B, const float* x, size_t x_stride, const float* norm_w, float eps,
                              float* xp, size_t xp_floats, const float* bias, const float* residual,
                              float* y, size_t y_stride, float* part, size_t part_floats,
                              cudaStream_t s);
// qmatmul_umma.cu: the same product on the 5th-generation tensor cores
// (tcgen05.mma, TMEM accumulators) for 1..64 quantized inputs.
bool qmatmul_umma_takes(int dtype, int cols, int B, size_t xp_floats);
minq_status launch_qmatmul_umma(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                                int B, const float* x, size_t x_stride, const float* norm_w,
                                float eps, float* xp, size_t xp_floats, const float* bias,
                                const float* residual, float* y, size_t y_stride, float* part,
                                size_t part_floats, cudaStream_t s);
minq_status launch_embed_batch(const float* embed, const uint32_t* d_tok, size_t vocab, int hidden,
                               int B, float* x, cudaStream_t s);
// argmax of each of the B rows of x [B][n]; scratch: 32 u64 per row.
minq_status launch_argmax_rows(const float* x, size_t n, int B, uint32_t* out,
                               unsigned long long* scratch, cudaStream_t s);

// attention.cu
size_t attn_workspace_bytes(size_t batch, size_t nh, size_t len, size_t hd_max);
// Exact workspace of one launch_attention call over `batch` entries whose
// longest history is size_len (head_major: the model's cache layout with
// 16-byte aligned K/V), 0 when it needs no split partials.
size_t attn_workspace_need(size_t batch, int nh, int nkv, int hd, int size_len, bool head_major);
minq_status launch_attention(const float* q, const float* k, const float* v, size_t batch,
                             int nh, int nkv, int hd, int len, size_t seq_stride,
                             size_t head_stride, size_t pos_stride, float* out, void* ws,
                             size_t ws_bytes, cudaStream_t s, const int* d_pos = nullptr,
                             int cap_len = 0, bool record_status = true, int len_step = 0,
                             int* status_word = nullptr);
// record_status = false: bounded-wait timeouts are not recorded (and the
// lazily allocated device status word is never touched); status_word, when
// set, replaces that allocated word as the place timeouts are recorded
// (minq_attend_static's file-scope word). len_step > 0
// (host positions only): entry b attends over len + b * len_step positions,
// e.g. the tokens of a prompt chunk over one cache (seq_stride 0).
// attn_prefill_tc.cu: causal attention of T prompt tokens at positions
// p0 .. p0 + T - 1 over a head-major layer cache (kv head h at
// k + h * head_stride, [position][hd]) that already holds their keys, on
// the tensor cores (tcgen05 kind::tf32, hi / lo split operands). q, out:
// [T][nh][hd]. workspace: prefill_attention_workspace(T, nh, nkv, hd) bytes.
bool prefill_attention_supported(int nh, int nkv, int hd);
size_t prefill_attention_workspace(int T, int nh, int nkv, int hd);
minq_status launch_prefill_attention(const float* q, const float* kc, const float* vc,
                                     size_t head_stride, int p0, int T, int nh, int nkv, int hd,
                                     float* out, void* ws, size_t ws_bytes, cudaStream_t s,
                                     int* status_word = nullptr);
minq_status launch_rope_append(const float* q_in, const float* k_in, const float* v_in,
                               size_t q_in_bstride, size_t kv_in_bstride, const float* q_norm,
                               const float* k_norm, float eps, const float* cos_t,
                               const float* sin_t, size_t batch, int nh, int nkv, int hd,
                               int pos, float* q_out, float* k_cache, float* v_cache,
                               size_t seq_stride, size_t head_stride, size_t pos_stride,
                               cudaStream_t s, const int* d_pos = nullptr, int pos_step = 0);
// pos_step: entry b is rotated and appended at position pos + b * pos_step.

// glue.cu
minq_status launch_embed(const float* embed, const uint32_t* d_tok, size_t vocab, int hidden,
                         float* x, cudaStream_t s);
minq_status launch_rmsnorm(const float* x, const float* w, float eps, int n, float* out,
                           cudaStream_t s);
minq_status launch_epilogue(const float* acc, const float* bias, const float* residual, float* y,
                            size_t n, cudaStream_t s);
minq_status launch_swiglu(const float* g, const float* u, float* h, size_t n, cudaStream_t s);
minq_status launch_advance_pos(int* pos, int by, cudaStream_t s);
// sampler.cu: the device a sampler was created on
int sampler_device(const minq_sampler* s);
// per-row negative log-likelihood (ppl.rs:30-35) of logits [rows][V] at
// targets[rows] (device), into out[rows] (f64)
minq_status launch_nll_rows(const float* logits, size_t V, int rows, const uint32_t* targets,
                            double* out, cudaStream_t s);

}  // namespace minq
