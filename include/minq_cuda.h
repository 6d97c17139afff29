/*
 * minq_cuda.h — C ABI of the B200 (sm_100a) implementation of minq's
 * KV-cached forward path.
 *
 * The reference (kn1g78/minq) is a Rust crate with no FFI; every entry point
 * below replaces one Rust function on the hot path and is what a thin Rust
 * FFI crate (`minq-cuda-sys`) would bind: an `extern "C"` block declaring
 * these functions, called from `Linear::matvec` and `Model::forward` when
 * the crate is built with the CUDA backend.
 *
 * Conventions
 *  - Every function returns a minq_status; on error, minq_last_error()
 *    returns a thread-local message (the text of the MinqError variant the
 *    reference would have produced, error.rs:5-28).
 *  - "device" pointers are CUDA global memory on the current device; "host"
 *    pointers are ordinary (pageable or pinned) host memory.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream). Op-level calls are asynchronous on that stream; model-level
 *    calls (minq_forward, minq_generate) are synchronous for the caller, like
 *    the Rust functions they replace.
 *  - Handles are not thread-safe; use one model/cache per host thread.
 *  - No entry point falls back to a CPU path: without a usable CUDA device
 *    every compute call returns MINQ_ERR_CUDA.
 */
#ifndef MINQ_CUDA_H_
#define MINQ_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MINQ_ABI_VERSION 1

/* error.rs:5-28 MinqError variants, plus the device-side failures. */
typedef enum minq_status {
  MINQ_OK = 0,
  MINQ_ERR_IO = 1,      /* MinqError::Io */
  MINQ_ERR_SHAPE = 2,   /* MinqError::Shape */
  MINQ_ERR_FORMAT = 3,  /* MinqError::Format */
  MINQ_ERR_MODEL = 4,   /* MinqError::Model */
  MINQ_ERR_CUDA = 5,    /* CUDA runtime / launch failure */
  MINQ_ERR_NCCL = 6,    /* NCCL failure (tensor-parallel decode) */
  MINQ_ERR_TIMEOUT = 7, /* a bounded device or collective wait gave up */
  MINQ_ERR_ARG = 8      /* null pointer / invalid enum */
} minq_status;

/* Storage tags of the .minq format (format.rs:37-39). */
typedef enum minq_dtype { MINQ_F32 = 0, MINQ_Q8_0 = 1, MINQ_Q4_0 = 2 } minq_dtype;

/* ModelConfig (model.rs:29-45). `dtype` is the storage tag of the file. */
typedef struct minq_config {
  uint64_t hidden_size;
  uint64_t intermediate_size;
  uint64_t n_layers;
  uint64_t n_heads;
  uint64_t n_kv_heads;
  uint64_t head_dim;
  uint64_t vocab_size;
  uint64_t max_seq_len;
  float rope_theta;
  float rms_norm_eps;
  int32_t has_qkv_bias;
  int32_t dtype;
} minq_config;

/* GenStats (engine.rs:11-27). */
typedef struct minq_gen_stats {
  uint64_t prompt_tokens;
  uint64_t gen_tokens;
  double prefill_secs;
  double decode_secs;
} minq_gen_stats;

/* PplResult (ppl.rs:16-27). */
typedef struct minq_ppl_result {
  uint64_t total_tokens;     /* tokens in the input sequence */
  uint64_t scored_positions; /* positions that contributed to the mean */
  double mean_nll;           /* mean cross-entropy (natural log) */
  double ppl;                /* exp(mean_nll) */
} minq_ppl_result;

typedef struct minq_model minq_model;
typedef struct minq_cache minq_cache;
typedef struct minq_sampler minq_sampler;

/* Engine::generate's `on_token` callback (engine.rs:56); a non-zero return
 * aborts generation and is reported as MINQ_ERR_MODEL (engine.rs:73). */
typedef int (*minq_token_cb)(uint32_t token, void* user);

/* eval_ppl's `on_window(done, total, cumulative_ppl)` progress callback
 * (ppl.rs:49), called after each window; cumulative_ppl is NaN while no
 * position has been scored. */
typedef void (*minq_ppl_window_cb)(size_t done, size_t total, double cumulative_ppl, void* user);

const char* minq_last_error(void);
int minq_abi_version(void);
/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads); a diagnostic for benchmarks. No reference
 * counterpart. */
uint64_t minq_kernel_launches(void);

/* Synchronise the current device and report whether any bounded
 * device-side wait (TMA pipeline barriers) gave up since the last check:
 * MINQ_ERR_TIMEOUT if so (and clear it), else MINQ_OK. minq_forward and
 * minq_generate check this themselves. */
minq_status minq_device_status(void);

/* Kernel timer (diagnostic; no reference counterpart). Between start and
 * stop, every launch of the named kernel family ("qmatvec", "f32_matvec",
 * "attention") is bracketed by CUDA events on its own stream. stop()
 * synchronises and returns the number of timed launches, their summed
 * device time in milliseconds and their summed algorithmic bytes (weights
 * or K/V read plus vectors read and written). */
minq_status minq_kernel_timer_start(const char* family);
minq_status minq_kernel_timer_stop(uint64_t* launches, double* total_ms, double* bytes);

/* ---------------------------------------------------------------------- */
/* Quantized blocks (quantize.rs)                                          */

/* quantize_q8_0 / quantize_q4_0 (quantize.rs:78,120) on the GPU; device x
 * [n] -> device out [n/32 * {36,20}] bytes, bit-identical to the reference.
 * n % 32 != 0 -> MINQ_ERR_SHAPE (quantize.rs:67-75). */
minq_status minq_quantize(minq_dtype dtype, const float* x, size_t n, void* out, void* stream);

/* dequantize_q8_0 / dequantize_q4_0 (quantize.rs:99,146); device in/out. */
minq_status minq_dequantize(minq_dtype dtype, const void* blocks, size_t nbytes, float* out,
                            size_t n_out, void* stream);

/* QuantizedTensor::matvec (quantize.rs:215-249): y[rows] = W[rows, cols] x.
 * `blocks` is the reference's row-major block layout, device memory.
 * x_len != cols -> MINQ_ERR_SHAPE (quantize.rs:216-222). */
minq_status minq_qmatvec(minq_dtype dtype, const void* blocks, size_t rows, size_t cols,
                         const float* x, size_t x_len, float* y, void* stream);

/* QuantizedTensor::matvec (quantize.rs:215-249) applied to `batch`
 * independent inputs at once, as the reference's per-sequence loop over
 * Linear::matvec (model.rs:57) would: y[b] = W x[b] for b < batch (1..64).
 * x [batch][cols] and y [batch][rows] are device f32, `blocks` the
 * row-major block layout (16-byte aligned). From 2 inputs on the product
 * runs on the tensor cores (tcgen05, f32 accumulation of exact weight codes
 * times a two-part bf16 split of x). `workspace` (device, 16-byte aligned)
 * holds minq_qmatmul_workspace_bytes(batch, rows, cols) bytes. Errors as
 * minq_qmatvec, plus MINQ_ERR_ARG for batch outside 1..64 or a small
 * workspace. */
size_t minq_qmatmul_workspace_bytes(size_t batch, size_t rows, size_t cols);
minq_status minq_qmatmul(minq_dtype dtype, const void* blocks, size_t rows, size_t cols,
                         const float* x, size_t batch, float* y, void* workspace,
                         size_t workspace_bytes, void* stream);

/* tensor::matvec (tensor.rs:181-192) for a dense f32 [rows, cols] weight. */
minq_status minq_matvec_f32(const float* w, size_t rows, size_t cols, const float* x,
                            size_t x_len, float* y, void* stream);

/* sampler::argmax (sampler.rs:10-17): total_cmp order, ties to the lowest
 * index. Device logits [n] -> device *out. */
minq_status minq_argmax(const float* logits, size_t n, uint32_t* out, void* stream);

/* ---------------------------------------------------------------------- */
/* Decode attention (model.rs:223-248 `attend`, plus the RoPE / q-k norm /  */
/* cache append that precede it in forward_token, model.rs:291-303)         */

/* Bytes of device workspace minq_attn_decode / minq_attend need for up to
 * `max_len` attended positions (any head_dim <= 256). */
size_t minq_attn_workspace_bytes(size_t batch, size_t n_heads, size_t max_len);

/* One decode-attention step for `batch` independent sequences at the same
 * position `pos`:
 *   q      [batch, n_heads, head_dim]     pre-RoPE query (left unchanged;
 *                                         the rotated copy lives in the
 *                                         workspace)
 *   k_new  [batch, n_kv, head_dim]        pre-RoPE key of this position
 *   v_new  [batch, n_kv, head_dim]
 *   q_norm, k_norm  [head_dim] or NULL    Qwen3 per-head RMSNorm gains
 *   rope_cos, rope_sin [>pos, head_dim/2] tables built like RopeTables::new
 *   k_cache, v_cache  cache of sequence b, kv-head h, position t at
 *                     element b*seq_stride + h*head_stride + t*pos_stride
 *                     (the reference's LayerCache layout is head_stride =
 *                     head_dim, pos_stride = n_kv*head_dim)
 *   out    [batch, n_heads, head_dim]
 * The rotated key and the value are appended at position `pos`, then every
 * query head attends over positions 0..=pos. `workspace` (device) must hold
 * minq_attn_workspace_bytes(batch, n_heads, pos+1) bytes. */
minq_status minq_attn_decode(const float* q, const float* k_new, const float* v_new,
                             const float* q_norm, const float* k_norm, float eps,
                             const float* rope_cos, const float* rope_sin, size_t batch,
                             size_t n_heads, size_t n_kv, size_t head_dim, size_t pos,
                             float* k_cache, float* v_cache, size_t seq_stride,
                             size_t head_stride, size_t pos_stride, float* out, void* workspace,
                             size_t workspace_bytes, void* stream);

/* attend() alone (no RoPE / append) over a position-major history
 * k, v [len, n_kv*head_dim] for one query q [n_heads*head_dim]; device
 * pointers. Unit-parity entry for model.rs:223-248. */
minq_status minq_attend(const float* q, const float* k, const float* v, size_t len,
                        size_t n_heads, size_t n_kv, size_t head_dim, float* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Causal attention of a prompt chunk, the reference's prompt loop
 * (model.rs:259-268 -> forward_token's attend, model.rs:223-248, one call per
 * token) done for n_tokens tokens at once: token t (position p0 + t) attends
 * over positions 0..=p0+t of a head-major layer cache whose positions
 * 0..p0+n_tokens-1 already hold every key and value, the chunk's own
 * included (kv head h at k_cache + h*head_stride, [position][head_dim]).
 *   q    [n_tokens, n_heads, head_dim]   RoPE'd queries
 *   out  [n_tokens, n_heads, head_dim]
 * Runs on the tensor cores (tcgen05 kind::tf32 with hi/lo split operands,
 * f32 accumulation: about the f32 arithmetic of the reference's dot
 * products). head_dim 64 or 128 (else MINQ_ERR_SHAPE); q, k, v, out
 * 16-byte aligned and head_stride a multiple of 4 (else MINQ_ERR_ARG).
 * `workspace` (device) holds minq_attn_prefill_workspace_bytes(n_tokens,
 * n_heads, n_kv, head_dim) bytes (0: none needed). */
size_t minq_attn_prefill_workspace_bytes(size_t n_tokens, size_t n_heads, size_t n_kv,
                                         size_t head_dim);
minq_status minq_attend_prefill(const float* q, const float* k_cache, const float* v_cache,
                                size_t head_stride, size_t p0, size_t n_tokens, size_t n_heads,
                                size_t n_kv, size_t head_dim, float* out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* minq_attend without a workspace argument: the split-KV scratch is a
 * 32 MiB array inside the library, so the call allocates no device memory.
 * No reference counterpart: added for callers that cannot allocate or own
 * device memory (a host language binding without a device allocator, a
 * real-time thread that must not take cudaMalloc's implicit
 * synchronisation). Limit: n_heads * ceil(len/32) * (head_dim+2) * 4 + 256
 * bytes <= 32 MiB, else MINQ_ERR_ARG and nothing is launched. The first
 * call on each device takes the scratch's address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * Calls that may overlap on the GPU (other streams, other host threads)
 * share the one scratch and race: order them on one stream or with events.
 * Nothing in the scratch needs to start at zero. A bounded device-side
 * wait that times out inside this call is recorded in a second file-scope
 * word, which minq_attend_static_status (and minq_device_status) report as
 * MINQ_ERR_TIMEOUT and clear. head_dim > 256 or n_heads > 4096: MINQ_ERR_SHAPE
 * as in minq_attend. */
minq_status minq_attend_static(const float* q, const float* k, const float* v, size_t len,
                               size_t n_heads, size_t n_kv, size_t head_dim, float* out,
                               void* stream);

/* Synchronises the current device, then reads and clears the timeout word of
 * minq_attend_static: MINQ_OK, or MINQ_ERR_TIMEOUT when a call since the last
 * read left `out` incomplete. Allocates nothing. */
minq_status minq_attend_static_status(void);

/* ---------------------------------------------------------------------- */
/* Model (model.rs:88-98, assemble :522-574, load_minq :711-715)           */

/* load_minq: parse a .minq file (format.rs:149-277) and upload it to the
 * current device. The file is mapped read-only and indexed in place (the
 * reader's length, shape and tag checks; MINQ_ERR_FORMAT / MINQ_ERR_IO as
 * read_minq), then each tensor goes from the mapping through two pinned
 * staging buffers to the device on a copy stream. */
minq_status minq_model_load(const char* path, minq_model** out);

/* Builder mirroring assemble(config, get): create, add named tensors (host
 * or device data in the .minq record encoding), then finish, which validates
 * the geometry exactly like assemble and builds the RoPE tables. */
minq_status minq_model_new(const minq_config* cfg, minq_model** out);
minq_status minq_model_add_tensor(minq_model* m, const char* name, minq_dtype tag,
                                  size_t ndim, const uint64_t* shape, const void* data,
                                  size_t nbytes, int data_on_device);
minq_status minq_model_finish(minq_model* m);
minq_status minq_model_config(const minq_model* m, minq_config* out);
/* Device bytes held by the model's weights (the per-token weight traffic). */
minq_status minq_model_weight_bytes(const minq_model* m, uint64_t* out);
void minq_model_free(minq_model* m);

/* Tensor-parallel decode over `world` GPUs (one process or thread per GPU,
 * each holding the whole model): minq_tp_unique_id (on one rank) makes the
 * NCCL id (128 bytes) that the caller hands to every rank; minq_tp_init then
 * keeps this rank's query / kv heads (q|k|v rows, o_proj columns) and
 * intermediate rows (gate/up rows, down_proj columns) and joins the NCCL
 * communicator. Afterwards minq_forward / minq_decode_steps (called by every
 * rank with the same tokens, in the same order) all-reduce the o_proj and
 * down_proj partial sums (2 per layer, hidden_size floats each); caches
 * created afterwards hold this rank's kv heads. Requires quantized
 * projections and n_heads, n_kv_heads divisible by world, intermediate_size
 * by 32 * world. */
minq_status minq_tp_unique_id(void* id_out);
minq_status minq_tp_init(minq_model* m, int rank, int world, const void* unique_id);

/* KVCache::new / reset (model.rs:117-130). The cache is preallocated in HBM
 * for `max_seq` positions (0 = config.max_seq_len) and `batch` independent
 * sequences (1 for the reference's single-sequence API). */
minq_status minq_cache_new(minq_model* m, size_t batch, size_t max_seq, minq_cache** out);
minq_status minq_cache_reset(minq_cache* c);
minq_status minq_cache_len(const minq_cache* c, size_t* out);
/* Write / read positions [start, start+n) of one layer, sequence 0, in the
 * reference's LayerCache layout ([n, n_kv*head_dim] f32, K post-RoPE), host
 * memory. Writing past the current length extends it (the reference's
 * public `LayerCache` fields allow the same pre-fill, model.rs:103-114).
 * minq_cache_set_len sets the length after a pre-fill of every layer. */
minq_status minq_cache_write(minq_cache* c, size_t layer, size_t start, size_t n,
                             const float* k, const float* v);
minq_status minq_cache_read(const minq_cache* c, size_t layer, size_t start, size_t n, float* k,
                            float* v);
/* minq_cache_write from device memory (the same [n, n_kv*head_dim] layout,
 * this rank's kv heads after minq_tp_init): the long-context pre-fill. */
minq_status minq_cache_write_device(minq_cache* c, size_t layer, size_t start, size_t n,
                                    const float* d_k, const float* d_v);
minq_status minq_cache_set_len(minq_cache* c, size_t len);
/* Frees the cache. A model freed first releases the device memory of its
 * caches still open; their handles then stay valid only for this call. */
void minq_cache_free(minq_cache* c);

/* Model::forward (model.rs:254-270): run `tokens` (host) through the model,
 * appending to the cache; writes the last token's logits to `logits_out`
 * (host, vocab_size floats, or NULL) and its argmax to `argmax_out` (host,
 * or NULL). Empty input -> MINQ_ERR_MODEL "empty token sequence"; a position
 * at max_seq_len -> MINQ_ERR_MODEL "sequence exceeds max_seq_len (N)";
 * token >= vocab -> MINQ_ERR_SHAPE. n > 1 runs the batched prefill path;
 * the cache and last logits match n single-token calls. */
minq_status minq_forward(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                         float* logits_out, uint32_t* argmax_out);

/* Batched decode step for the `batch` sequences of a cache created with
 * minq_cache_new(m, batch, ...) (batch <= 64): `tokens` (host, n == batch
 * ids) holds one token per sequence; every sequence runs Model::forward_token
 * (model.rs:273-318) at the cache's common position, which then advances by
 * one. `logits_out` (host, batch x vocab floats, or NULL) and `argmax_out`
 * (host, batch ids, or NULL) get each sequence's results. Replaces the
 * reference's per-sequence loop over Model::forward (64 independent
 * sequences, data-sharded by the caller); the weights are read once per step
 * for all sequences. Errors as minq_forward, plus MINQ_ERR_ARG when n !=
 * batch. */
minq_status minq_forward_batch(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                               float* logits_out, uint32_t* argmax_out);

/* Prompts of the `batch` sequences of a batched cache (the reference's
 * Model::forward prompt loop, model.rs:254-270, run per sequence): sequence b
 * takes tokens[b*n .. b*n + n - 1] (host) at the cache's common positions
 * len .. len + n - 1. All but the last token of each sequence go through the
 * chunked prefill (64 tokens of one sequence per pass: projections and causal
 * attention on the tensor cores), the last tokens as one batched step whose
 * logits (`logits_out`, host, batch x vocab floats, or NULL) and argmax
 * (`argmax_out`, host, batch ids, or NULL) are returned. The cache and the
 * outputs match n calls of minq_forward_batch with column i of `tokens`.
 * Errors as minq_forward_batch. */
minq_status minq_prefill_batch(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                               float* logits_out, uint32_t* argmax_out);

/* Greedy continuation of a batched cache on the device: n_steps batched
 * steps, each feeding every sequence its previous argmax (no host
 * synchronisation); `d_tokens_out` (device, n_steps x batch ids, or NULL). */
minq_status minq_forward_batch_device(minq_model* m, minq_cache* c, size_t n_steps,
                                      uint32_t* d_tokens_out);

/* Same as minq_forward with device-resident token ids and outputs on the
 * model's stream (no host synchronisation): used to measure the kernels
 * without host copies and to chain decode steps. */
minq_status minq_forward_device(minq_model* m, minq_cache* c, const uint32_t* d_tokens,
                                size_t n, float* d_logits, uint32_t* d_argmax);

/* Greedy decode continuation on the device (the decode loop of
 * engine.rs:71-79 with Sampler::greedy, without the host in the loop):
 * n_steps forward passes on the model's stream, each consuming the argmax
 * left by the previous minq_forward / minq_decode_steps step and appending
 * to the cache. No host synchronisation; `d_tokens_out` (device, n_steps
 * ids, or NULL) receives the generated ids. The cache must be non-empty. */
minq_status minq_decode_steps(minq_model* m, minq_cache* c, size_t n_steps,
                              uint32_t* d_tokens_out);

/* Replay each single-token step as a CUDA graph captured once per cache
 * (default on; MINQ_GRAPHS=0 in the environment turns the default off), or
 * launch its kernels one by one (needed by minq_kernel_timer_*). */
minq_status minq_model_set_graphs(minq_model* m, int enabled);

/* Engine::generate with Sampler::greedy (engine.rs:52-88): prefill the
 * prompt, then up to max_tokens greedy steps; `on_token` may be NULL;
 * `stop_tokens` (host, n_stop) end generation after reporting the token. */
minq_status minq_generate(minq_model* m, const uint32_t* prompt, size_t n_prompt,
                          size_t max_tokens, const uint32_t* stop_tokens, size_t n_stop,
                          minq_token_cb on_token, void* user, uint32_t* tokens_out,
                          minq_gen_stats* stats);

/* Model::forward_full_states (model.rs:337-424): the hidden state of every
 * position of `tokens` (host, n ids) after the last decoder layer, before the
 * final RMSNorm, into `states_out` (host, n x hidden_size floats, or NULL to
 * run the sweep only). Runs on a scratch cache of n positions, chunk by chunk
 * (64 positions per pass, causal), and leaves no state behind. Empty input ->
 * MINQ_ERR_MODEL "empty token sequence"; n > max_seq_len -> MINQ_ERR_MODEL
 * "sequence exceeds max_seq_len (N)"; token >= vocab -> MINQ_ERR_SHAPE; a
 * model the chunked sweep does not take (tensor-parallel, f32 q|k|v or
 * gate/up projections, dimensions not multiples of 32) -> MINQ_ERR_SHAPE. */
minq_status minq_forward_full_states(minq_model* m, const uint32_t* tokens, size_t n,
                                     float* states_out);

/* eval_ppl (ppl.rs:44-103): split `tokens` (host, n ids) into
 * non-overlapping windows of `context` tokens, sweep each window causally
 * (as minq_forward_full_states), and score position t in 1 .. len - 2 of a
 * window by the negative log-likelihood of window[t + 1] under the lm_head
 * logits of its final-RMSNorm'd state (log-sum-exp in f64, ppl.rs:30-35),
 * summed in f64 in position order. `on_window` (or NULL) is called after
 * each window. n < 3, context < 3, context > max_seq_len, or no scorable
 * position -> MINQ_ERR_MODEL with the reference's messages; token >= vocab
 * -> MINQ_ERR_SHAPE when its window is reached; shapes the sweep does not
 * take -> MINQ_ERR_SHAPE. */
minq_status minq_eval_ppl(minq_model* m, const uint32_t* tokens, size_t n, size_t context,
                          minq_ppl_window_cb on_window, void* user, minq_ppl_result* out);

/* Sampler::new (sampler.rs:32-40) on the current CUDA device: temperature
 * (<= 0: greedy), top_k (0: off), top_p (>= 1: off) and the StdRng seed
 * (rand 0.8 StdRng::seed_from_u64: ChaCha12 keyed by PCG32 outputs), whose
 * state lives in device memory and advances once per non-greedy draw. */
minq_status minq_sampler_new(float temperature, size_t top_k, float top_p, uint64_t seed,
                             minq_sampler** out);
void minq_sampler_free(minq_sampler* s);

/* Sampler::sample (sampler.rs:47-109) on device logits (n floats) into
 * d_token (device, one id), enqueued on `stream` (cudaStream_t, NULL: the
 * legacy default stream) with no host synchronisation. Greedy samplers take
 * the argmax (total_cmp, ties low). Otherwise softmax(logits / temperature),
 * then one uniform draw: over the whole distribution without filters, else
 * over the top_k most probable (ties at the boundary by lower index; the
 * reference leaves their order unspecified) cut at the top_p cumulative
 * mass, renormalised. Probabilities use the f64 exponential rounded to f32
 * and f64 running sums, so a draw can differ from the reference's only when
 * the uniform falls within rounding of a boundary, and then by a neighbouring
 * token. n == 0 -> token 0; n > 4194304 -> MINQ_ERR_ARG. */
minq_status minq_sampler_sample_device(minq_sampler* s, const float* d_logits, size_t n,
                                       uint32_t* d_token, void* stream);

/* The same with host logits and a host token (synchronous). */
minq_status minq_sampler_sample(minq_sampler* s, const float* logits, size_t n,
                                uint32_t* token_out);

/* Diagnostic: the sampler's next n raw StdRng outputs (RngCore::next_u32),
 * advancing its state; n <= 2^20. No reference counterpart. */
minq_status minq_sampler_rng_u32(minq_sampler* s, size_t n, uint32_t* out);

/* Engine::generate (engine.rs:52-88) with the given Sampler: prefill the
 * prompt, then up to max_tokens steps, each token drawn on the device from
 * the step's logits (no logits copy to the host; 4 bytes come back per token
 * for on_token and the stop check). The sampler must live on the model's
 * device. Errors as minq_generate. */
minq_status minq_generate_sampled(minq_model* m, minq_sampler* s, const uint32_t* prompt,
                                  size_t n_prompt, size_t max_tokens,
                                  const uint32_t* stop_tokens, size_t n_stop,
                                  minq_token_cb on_token, void* user, uint32_t* tokens_out,
                                  minq_gen_stats* stats);

/* The model's CUDA stream (cudaStream_t as void*). */
void* minq_model_stream(minq_model* m);

/* Failure injection for tests (no reference counterpart): make a bounded
 * device-side wait of the next decode-megakernel step run out by moving its
 * target out of reach on the host. what = 0: the per-head attention merge
 * counters; 1: the grid barrier. That step then returns MINQ_ERR_TIMEOUT
 * after the wait limit (1 s) with the megakernel's barrier state reset, and
 * later steps run normally (the cache of the failed step should be reset).
 * MINQ_ERR_ARG when the model does not use the decode megakernel. */
minq_status minq_debug_inject_timeout(minq_model* m, int what);

#ifdef __cplusplus
}
#endif

#endif /* MINQ_CUDA_H_ */
