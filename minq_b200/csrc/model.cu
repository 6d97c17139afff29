// Device-resident model, KV cache and the KV-cached forward step
// (model.rs:88-318, engine.rs:52-88) behind the C ABI of include/minq_cuda.h.
//
// Layout in HBM:
//   * weights keep the .minq encoding: quantized matrices in the reference's
//     row-major AoS block layout; q/k/v of a layer are concatenated into one
//     [qd + 2*kvd, H] matrix when they share a quantized dtype, so one matvec
//     launch covers all three projections (plus the concatenated bias);
//   * the tied lm_head aliases the f32 embedding table (no clone, unlike
//     model.rs:564);
//   * the KV cache is preallocated per layer as [batch][n_kv][max_seq][hd]
//     f32 (head-major: one contiguous stream per KV head for decode
//     attention), K stored post-RoPE like LayerCache (model.rs:100-106);
//   * RoPE cos/sin tables [max_seq_len, hd/2] are built on the host with the
//     reference's f32 expression and glibc (model.rs:170-186) and uploaded.
//
// Execution: one decode step is ~5 kernels per layer, each launched with
// programmatic dependent launch. The step reads its position from a device
// counter (advanced by the step itself), so it is captured once per cache as
// a CUDA graph and replayed for every token; prefill replays the no-logits
// graph token by token.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "decode_mk.h"
#include "nccl_dl.h"
#include "kernels.h"
#include "minq_format.h"

namespace minq {

struct DevTensor {
  int tag = -1;
  std::vector<uint64_t> shape;
  void* ptr = nullptr;
  size_t nbytes = 0;
};

struct DevLinear {
  int tag = -1;  // MINQ_F32 / MINQ_Q8_0 / MINQ_Q4_0; -1 absent
  uint64_t rows = 0, cols = 0;
  const void* ptr = nullptr;
  size_t nbytes = 0;
  CUtensorMap tm;     // 2-D TMA map for the TMA-fed matvec (when tm_ok)
  bool tm_ok = false;
};

struct DevLayer {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  DevLinear q, k, v, o, gate, up, down;
  DevLinear qkv;                 // fused q|k|v (tag -1 when not fused)
  float* bias_qkv = nullptr;     // [qd + 2*kvd] when any bias exists
  const float* q_bias = nullptr;
  const float* k_bias = nullptr;
  const float* v_bias = nullptr;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
};

}  // namespace minq

using minq::DevLayer;
using minq::DevLinear;
using minq::DevTensor;

struct minq_model {
  minq_config cfg{};
  int device = 0;
  // tensor parallelism (minq_tp_init): this rank's query / kv heads and
  // intermediate rows; the full counts on a single GPU
  int tp_rank = 0, tp_world = 1;
  void* tp_comm = nullptr;  // ncclComm_t
  minq::TpAr tpar;          // peer-memory all-reduce (NCCL when off)
  int nh_l = 0, nkv_l = 0;
  uint64_t I_l = 0;
  cudaStream_t stream = nullptr;
  bool finished = false;
  bool use_graphs = true;
  std::map<std::string, DevTensor> pending;
  std::vector<void*> allocs;
  std::set<minq_cache*> caches;  // live caches: freed with the model if still open
  // assembled
  const float* embed = nullptr;
  std::vector<DevLayer> layers;
  const float* final_norm = nullptr;
  DevLinear lm_head;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  std::string shape_error;  // reported by forward as MinqError::Shape
  uint64_t weight_bytes = 0;
  // activation scratch (single sequence)
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *q_rot = nullptr, *att = nullptr;
  float *hbuf = nullptr, *gbuf = nullptr, *ubuf = nullptr, *tmp = nullptr, *logits = nullptr;
  unsigned long long* argmax_part = nullptr;
  int argmax_cap = 0;
  uint32_t* d_tok = nullptr;     // the step's input token and, after it, its argmax
  uint32_t* d_tokens = nullptr;  // staged prompt
  size_t d_tokens_cap = 0;
  // decode megakernel (decode_mk.cu): set up at finish when the model fits it
  struct {
    bool ok = false;
    int dtype = 0, grid = 0, scratch = 0, nsplit = 0;
    size_t smem = 0;
    minq::MkMat qkv{}, o{}, gu{}, down{};
    minq::MkLayerPtrs* layers = nullptr;
    float* part = nullptr;
    unsigned* head_ctr = nullptr;
    unsigned* head_base = nullptr;
    unsigned long long* argmax_part = nullptr;
    unsigned long long* bar = nullptr;  // [0] counter, [1] base
    int* abort_flag = nullptr;
    uint2* xr = nullptr;       // residual stream exchange sites [2 n_layers][H] (one GPU)
    uint2** xr_dst = nullptr;  // device array {xr}
    unsigned* xr_epoch = nullptr;
  } mk;
};

struct minq_cache {
  minq_model* m = nullptr;
  size_t batch = 1, max_seq = 0, len = 0;
  float* k = nullptr;  // [n_layers][batch][n_kv][max_seq][hd]
  float* v = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* d_pos = nullptr;        // device copy of `len` read by graph-captured steps
  bool d_pos_valid = false;
  cudaGraphExec_t step[2] = {nullptr, nullptr};  // [0]: no logits, [1]: logits + argmax
  // activations of the batched step (minq_forward_batch), allocated on first use
  float* bx = nullptr;     // [batch][H] residual stream
  float* bqkv = nullptr;   // [batch][qd + 2 kvd]
  float* bq = nullptr;     // [batch][qd] RoPE'd queries
  float* batt = nullptr;   // [batch][qd]
  float* bh = nullptr;     // [batch][I]
  float* blog = nullptr;   // [batch][vocab]
  float* bxn = nullptr;    // prepared projection inputs: [batch][max(H, qd, I)] floats
  size_t bxn_floats = 0;
  float* bpart = nullptr;  // column-slice partials of the batched matvec
  size_t bpart_floats = 0;
  uint32_t* btok = nullptr;  // [batch] token ids
  uint32_t* barg = nullptr;  // [batch] argmax ids
  // activations of chunked prompt prefill (kPrefillChunk tokens of a batch-1
  // cache per pass), allocated on first use
  float* px = nullptr;     // [chunk][H]
  float* pqkv = nullptr;   // [chunk][qd + 2 kvd]
  float* pq = nullptr;     // [chunk][qd]
  float* patt = nullptr;   // [chunk][qd]
  float* ph = nullptr;     // [chunk][I]
  float* pxn = nullptr;    // prepared projection inputs
  size_t pxn_floats = 0;
  float* ppart = nullptr;  // column-slice partials
  size_t ppart_floats = 0;
  void* pws = nullptr;     // attention split partials
  size_t pws_bytes = 0;
  // perplexity scoring of a chunk: [chunk][vocab] logits, [chunk] f64 nll
  float* plog = nullptr;
  double* pnll = nullptr;
};

// The cache's device memory and graphs (its model's device current, stream idle).
static void cache_release_device(minq_cache* c) {
  for (cudaGraphExec_t g : c->step)
    if (g) cudaGraphExecDestroy(g);
  c->step[0] = c->step[1] = nullptr;
  cudaFree(c->k);
  cudaFree(c->v);
  cudaFree(c->ws);
  cudaFree(c->d_pos);
  for (void* b : {(void*)c->bx, (void*)c->bqkv, (void*)c->bq, (void*)c->batt, (void*)c->bh,
                  (void*)c->blog, (void*)c->bxn, (void*)c->bpart, (void*)c->btok,
                  (void*)c->barg, (void*)c->px, (void*)c->pqkv, (void*)c->pq, (void*)c->patt,
                  (void*)c->ph, (void*)c->pxn, (void*)c->ppart, c->pws, (void*)c->plog,
                  (void*)c->pnll})
    cudaFree(b);
}


namespace minq {

namespace {

minq_status dmalloc(minq_model* m, void** p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  m->allocs.push_back(*p);
  return MINQ_OK;
}

// Grows the staged-token buffer m->d_tokens to hold n ids. The old buffer is
// freed (after the model's stream has drained any copy or kernel that still
// reads it) and leaves m->allocs, so repeated calls on growing inputs keep
// one buffer, not every earlier one.
minq_status reserve_tokens(minq_model* m, size_t n) {
  if (n <= m->d_tokens_cap) return MINQ_OK;
  const size_t cap = std::max(n, 2 * m->d_tokens_cap);
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  void* old = m->d_tokens;
  if (old) {
    auto it = std::find(m->allocs.begin(), m->allocs.end(), old);
    if (it != m->allocs.end()) m->allocs.erase(it);
    MINQ_CUDA_TRY(cudaFree(old));
  }
  m->d_tokens = nullptr;
  m->d_tokens_cap = 0;
  void* p;
  MINQ_TRY(dmalloc(m, &p, cap * 4));
  m->d_tokens = static_cast<uint32_t*>(p);
  m->d_tokens_cap = cap;
  return MINQ_OK;
}

// RopeTables::new (model.rs:171-186): freq = 1 / theta^(2i/hd), angle =
// pos * freq, (sin, cos) = angle.sin_cos(), all in f32 through glibc. The
// calls go through volatile pointers so the host compiler neither folds nor
// fuses them into a different routine.
void build_rope_tables(uint64_t hd, uint64_t max_seq, float theta, std::vector<float>* cs,
                       std::vector<float>* sn) {
  float (*volatile powf_p)(float, float) = ::powf;
  float (*volatile sinf_p)(float) = ::sinf;
  float (*volatile cosf_p)(float) = ::cosf;
  const uint64_t half = hd / 2;
  cs->assign(max_seq * half, 0.0f);
  sn->assign(max_seq * half, 0.0f);
  std::vector<float> freq(half);
  for (uint64_t i = 0; i < half; ++i) {
    volatile float e = 2.0f * (float)i / (float)hd;
    freq[i] = 1.0f / powf_p(theta, e);
  }
  for (uint64_t pos = 0; pos < max_seq; ++pos) {
    for (uint64_t i = 0; i < half; ++i) {
      volatile float angle = (float)pos * freq[i];
      (*sn)[pos * half + i] = sinf_p(angle);
      (*cs)[pos * half + i] = cosf_p(angle);
    }
  }
}

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

minq_status need(minq_model* m, const std::string& name, DevTensor** out) {
  auto it = m->pending.find(name);
  if (it == m->pending.end()) return fail(MINQ_ERR_MODEL, "missing tensor `" + name + "`");
  *out = &it->second;
  return MINQ_OK;
}

minq_status get_linear(minq_model* m, const std::string& name, DevLinear* out) {
  DevTensor* t;
  MINQ_TRY(need(m, name, &t));
  if (t->tag == MINQ_F32 && t->shape.size() != 2)
    return fail(MINQ_ERR_MODEL, "tensor `" + name + "` must be 2-D, got " + shape_str(t->shape));
  out->tag = t->tag;
  out->rows = t->shape[0];
  out->cols = t->shape[1];
  out->ptr = t->ptr;
  out->nbytes = t->nbytes;
  return MINQ_OK;
}

minq_status get_vec(minq_model* m, const std::string& name, bool required, const float** out,
                    uint64_t* len) {
  auto it = m->pending.find(name);
  if (it == m->pending.end()) {
    if (required) return fail(MINQ_ERR_MODEL, "missing tensor `" + name + "`");
    *out = nullptr;
    return MINQ_OK;
  }
  const DevTensor& t = it->second;
  if (t.tag != MINQ_F32 || t.shape.size() != 1)
    return fail(MINQ_ERR_MODEL, "tensor `" + name + "` must be a 1-D f32 vector");
  *out = static_cast<const float*>(t.ptr);
  if (len) *len = t.shape[0];
  return MINQ_OK;
}

// Record the first geometry mismatch; the reference reports it as
// MinqError::Shape from the first matvec that sees it (quantize.rs:216-222,
// tensor.rs:182-188), so forward returns it rather than load.
void check_linear(minq_model* m, const DevLinear& l, uint64_t rows, uint64_t cols,
                  const char* what) {
  if (!m->shape_error.empty()) return;
  if (l.cols != cols)
    m->shape_error = std::string(l.tag == MINQ_F32 ? "matvec" : "quantized matvec") + ": " +
                     what + " has " + std::to_string(l.cols) + " cols vs input len " +
                     std::to_string(cols);
  else if (l.rows != rows)
    m->shape_error = std::string(what) + ": " + std::to_string(l.rows) + " rows, expected " +
                     std::to_string(rows);
}

void check_vec(minq_model* m, const float* p, uint64_t len, uint64_t want, const char* what) {
  if (!m->shape_error.empty() || !p) return;
  if (len != want)
    m->shape_error = std::string(what) + ": length " + std::to_string(len) + ", expected " +
                     std::to_string(want);
}

// Pre-encode the TMA tensor map of a quantized linear for its launch plan.
minq_status prepare_map(DevLinear* l, bool dual, bool norm) {
  if (l->tag != MINQ_Q8_0 && l->tag != MINQ_Q4_0) return MINQ_OK;
  if (l->cols % 128 != 0 || (uintptr_t)l->ptr % 16 != 0) return MINQ_OK;
  const QmvPlan t = plan_qmatvec_tma(l->tag, dual, l->rows, (int)l->cols, norm);
  MINQ_TRY(encode_qmatvec_map(l->ptr, l->rows, (int)l->cols, l->tag, t.nr, &l->tm));
  l->tm_ok = true;
  return MINQ_OK;
}

const CUtensorMap* map_of(const DevLinear& l) { return l.tm_ok ? &l.tm : nullptr; }

}  // namespace

// assemble (model.rs:522-574) on device tensors.
// Decide whether the batch-1 decode step runs as the megakernel and set it up
// (tensor maps for its tile plans, per-layer pointers, barrier state).
minq_status setup_megakernel(minq_model* m) {
  const char* env = std::getenv("MINQ_MEGAKERNEL");
  if (env && env[0] == '0') return MINQ_OK;
  const minq_config& c = m->cfg;
  // this rank's heads and intermediate rows (all of them on one GPU)
  const uint64_t H = c.hidden_size, I = m->I_l, hd = c.head_dim;
  const uint64_t nh = (uint64_t)m->nh_l, nkv = (uint64_t)m->nkv_l, qd = nh * hd, kvd = nkv * hd;
  if (m->tp_world > 1 && !m->tpar.on) return MINQ_OK;  // the megakernel needs the peer slots
  if (c.n_layers == 0 || nkv == 0 || nh % nkv != 0) return MINQ_OK;
  const uint64_t G = nh / nkv;
  if ((hd != 64 && hd != 128) || G > 8) return MINQ_OK;
  if (H % 128 || I % 128 || qd % 128) return MINQ_OK;
  if (m->lm_head.tag != MINQ_F32 || m->lm_head.cols != H) return MINQ_OK;
  const int dt = m->layers[0].o.tag;
  if (dt != MINQ_Q8_0 && dt != MINQ_Q4_0) return MINQ_OK;
  auto ok_lin = [&](const DevLinear& l) {
    return l.tag == dt && (uintptr_t)l.ptr % 16 == 0;
  };
  for (const DevLayer& L : m->layers)
    if (!ok_lin(L.qkv) || !ok_lin(L.o) || !ok_lin(L.gate) || !ok_lin(L.up) || !ok_lin(L.down))
      return MINQ_OK;
  const int grid = sm_count();
  auto& k = m->mk;
  k.dtype = dt;
  k.grid = grid;
  k.qkv = mk_plan_mat(dt, false, qd + 2 * kvd, H, grid);
  k.o = mk_plan_mat(dt, false, H, qd, grid);
  k.gu = mk_plan_mat(dt, true, I, H, grid);
  k.down = mk_plan_mat(dt, false, H, I, grid);
  for (const MkMat* mm : {&k.qkv, &k.o, &k.gu, &k.down})
    if (mm->rows == 0) return MINQ_OK;  // the consumer's row sums do not take the shape
  // history splits per kv head: up to one CTA each, as many as the merge
  // buffer in shared memory allows
  k.nsplit = std::max(1, grid / (int)nkv);
  if (const char* e = std::getenv("MINQ_MK_SPLITS"))  // at most this many splits per kv head
    if (std::atoi(e) > 0) k.nsplit = std::min(k.nsplit, std::atoi(e));
  for (;;) {
    k.scratch = (int)mk_scratch_bytes((int)H, (int)I, (int)qd, (int)G, (int)hd, k.nsplit);
    k.smem = mk_smem_bytes(k.scratch, (int)c.n_layers);
    if (k.smem != 0 || k.nsplit == 1) break;
    --k.nsplit;
  }
  if (k.smem == 0) return MINQ_OK;
  const size_t nl = c.n_layers;
  std::vector<MkLayerPtrs> lps(nl);
  for (size_t li = 0; li < nl; ++li) {
    const DevLayer& L = m->layers[li];
    auto u8 = [](const DevLinear& l) { return static_cast<const uint8_t*>(l.ptr); };
    lps[li] = MkLayerPtrs{u8(L.qkv), u8(L.o), u8(L.gate), u8(L.up), u8(L.down),
                          L.attn_norm, L.ffn_norm, L.bias_qkv, L.q_norm, L.k_norm};
  }
  void* p;
  MINQ_TRY(dmalloc(m, &p, lps.size() * sizeof(MkLayerPtrs)));
  k.layers = static_cast<MkLayerPtrs*>(p);
  MINQ_CUDA_TRY(cudaMemcpy(p, lps.data(), lps.size() * sizeof(MkLayerPtrs),
                           cudaMemcpyHostToDevice));
  MINQ_TRY(dmalloc(m, &p, nkv * k.nsplit * G * (hd + 2) * 4));
  k.part = static_cast<float*>(p);
  MINQ_TRY(dmalloc(m, &p, nkv * 4 + 4 + 2 * 8 + (size_t)grid * 8 + 64));
  k.bar = static_cast<unsigned long long*>(p);                         // 2 u64
  k.argmax_part = k.bar + 2;                                           // grid u64
  k.head_ctr = reinterpret_cast<unsigned*>(k.argmax_part + grid);      // nkv
  k.abort_flag = reinterpret_cast<int*>(k.head_ctr + nkv);             // 1
  k.head_base = reinterpret_cast<unsigned*>(k.abort_flag + 1);         // 1 (in the slack)
  MINQ_CUDA_TRY(cudaMemset(p, 0, nkv * 4 + 4 + 2 * 8 + (size_t)grid * 8 + 64));
  // the residual stream's exchange sites (value, epoch pairs) and epoch
  const size_t xr_bytes = 2 * nl * H * sizeof(uint2);
  MINQ_TRY(dmalloc(m, &p, xr_bytes + 256));
  MINQ_CUDA_TRY(cudaMemset(p, 0, xr_bytes + 256));
  k.xr = static_cast<uint2*>(p);
  k.xr_epoch = reinterpret_cast<unsigned*>(static_cast<char*>(p) + xr_bytes);
  MINQ_TRY(dmalloc(m, &p, sizeof(uint2*)));
  k.xr_dst = static_cast<uint2**>(p);
  MINQ_CUDA_TRY(cudaMemcpy(k.xr_dst, &k.xr, sizeof(uint2*), cudaMemcpyHostToDevice));
  k.ok = true;
  return MINQ_OK;
}

minq_status model_finish(minq_model* m) {
  const minq_config& c = m->cfg;
  if (c.head_dim % 2 != 0) return fail(MINQ_ERR_MODEL, "head_dim must be even (RoPE)");
  if (c.n_kv_heads == 0 || c.n_heads % c.n_kv_heads != 0)
    return fail(MINQ_ERR_MODEL, "n_heads must be a multiple of n_kv_heads");
  DevTensor* emb;
  MINQ_TRY(need(m, "model.embed_tokens.weight", &emb));
  if (emb->tag != MINQ_F32 || emb->shape.size() != 2)
    return fail(MINQ_ERR_MODEL, "model.embed_tokens.weight must be 2-D f32");
  m->embed = static_cast<const float*>(emb->ptr);
  const uint64_t H = c.hidden_size, hd = c.head_dim, qd = c.n_heads * hd,
                 kvd = c.n_kv_heads * hd, I = c.intermediate_size;
  if (emb->shape[1] != H && m->shape_error.empty())
    m->shape_error = "embedding width " + std::to_string(emb->shape[1]) + " != hidden_size";
  if (emb->shape[0] < c.vocab_size && m->shape_error.empty())
    m->shape_error = "embedding has " + std::to_string(emb->shape[0]) + " rows < vocab_size";
  m->layers.assign(c.n_layers, DevLayer());
  m->weight_bytes = 0;
  for (uint64_t i = 0; i < c.n_layers; ++i) {
    const std::string p = "model.layers." + std::to_string(i);
    DevLayer& L = m->layers[i];
    uint64_t n1 = 0, n2 = 0, nqb = 0, nkb = 0, nvb = 0, nqn = 0, nkn = 0;
    MINQ_TRY(get_vec(m, p + ".input_layernorm.weight", true, &L.attn_norm, &n1));
    MINQ_TRY(get_linear(m, p + ".self_attn.q_proj.weight", &L.q));
    MINQ_TRY(get_linear(m, p + ".self_attn.k_proj.weight", &L.k));
    MINQ_TRY(get_linear(m, p + ".self_attn.v_proj.weight", &L.v));
    MINQ_TRY(get_linear(m, p + ".self_attn.o_proj.weight", &L.o));
    MINQ_TRY(get_vec(m, p + ".self_attn.q_proj.bias", false, &L.q_bias, &nqb));
    MINQ_TRY(get_vec(m, p + ".self_attn.k_proj.bias", false, &L.k_bias, &nkb));
    MINQ_TRY(get_vec(m, p + ".self_attn.v_proj.bias", false, &L.v_bias, &nvb));
    MINQ_TRY(get_vec(m, p + ".self_attn.q_norm.weight", false, &L.q_norm, &nqn));
    MINQ_TRY(get_vec(m, p + ".self_attn.k_norm.weight", false, &L.k_norm, &nkn));
    MINQ_TRY(get_vec(m, p + ".post_attention_layernorm.weight", true, &L.ffn_norm, &n2));
    MINQ_TRY(get_linear(m, p + ".mlp.gate_proj.weight", &L.gate));
    MINQ_TRY(get_linear(m, p + ".mlp.up_proj.weight", &L.up));
    MINQ_TRY(get_linear(m, p + ".mlp.down_proj.weight", &L.down));
    check_vec(m, L.attn_norm, n1, H, "input_layernorm");
    check_linear(m, L.q, qd, H, "q_proj");
    check_linear(m, L.k, kvd, H, "k_proj");
    check_linear(m, L.v, kvd, H, "v_proj");
    check_vec(m, L.q_bias, nqb, qd, "q_proj.bias");
    check_vec(m, L.k_bias, nkb, kvd, "k_proj.bias");
    check_vec(m, L.v_bias, nvb, kvd, "v_proj.bias");
    check_vec(m, L.q_norm, nqn, hd, "q_norm");
    check_vec(m, L.k_norm, nkn, hd, "k_norm");
    check_linear(m, L.o, H, qd, "o_proj");
    check_vec(m, L.ffn_norm, n2, H, "post_attention_layernorm");
    check_linear(m, L.gate, I, H, "gate_proj");
    check_linear(m, L.up, I, H, "up_proj");
    check_linear(m, L.down, H, I, "down_proj");
    for (const DevLinear* l : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
      m->weight_bytes += l->nbytes;
    // Fuse q|k|v (same quantized dtype, consistent shapes) into one matrix.
    if (m->shape_error.empty() && L.q.tag != MINQ_F32 && L.q.tag == L.k.tag &&
        L.q.tag == L.v.tag) {
      void* buf;
      const size_t nb = L.q.nbytes + L.k.nbytes + L.v.nbytes;
      MINQ_TRY(dmalloc(m, &buf, nb));
      char* d = static_cast<char*>(buf);
      MINQ_CUDA_TRY(cudaMemcpyAsync(d, L.q.ptr, L.q.nbytes, cudaMemcpyDeviceToDevice, m->stream));
      MINQ_CUDA_TRY(cudaMemcpyAsync(d + L.q.nbytes, L.k.ptr, L.k.nbytes,
                                    cudaMemcpyDeviceToDevice, m->stream));
      MINQ_CUDA_TRY(cudaMemcpyAsync(d + L.q.nbytes + L.k.nbytes, L.v.ptr, L.v.nbytes,
                                    cudaMemcpyDeviceToDevice, m->stream));
      L.qkv.tag = L.q.tag;
      L.qkv.rows = qd + 2 * kvd;
      L.qkv.cols = H;
      L.qkv.ptr = buf;
      L.qkv.nbytes = nb;
      if (L.q_bias || L.k_bias || L.v_bias) {
        void* bb;
        MINQ_TRY(dmalloc(m, &bb, (qd + 2 * kvd) * 4));
        L.bias_qkv = static_cast<float*>(bb);
        MINQ_CUDA_TRY(cudaMemsetAsync(bb, 0, (qd + 2 * kvd) * 4, m->stream));
        if (L.q_bias)
          MINQ_CUDA_TRY(cudaMemcpyAsync(L.bias_qkv, L.q_bias, qd * 4, cudaMemcpyDeviceToDevice,
                                        m->stream));
        if (L.k_bias)
          MINQ_CUDA_TRY(cudaMemcpyAsync(L.bias_qkv + qd, L.k_bias, kvd * 4,
                                        cudaMemcpyDeviceToDevice, m->stream));
        if (L.v_bias)
          MINQ_CUDA_TRY(cudaMemcpyAsync(L.bias_qkv + qd + kvd, L.v_bias, kvd * 4,
                                        cudaMemcpyDeviceToDevice, m->stream));
      }
    }
    if (m->shape_error.empty()) {
      if (L.qkv.tag >= 0) MINQ_TRY(prepare_map(&L.qkv, false, true));
      MINQ_TRY(prepare_map(&L.o, false, false));
      MINQ_TRY(prepare_map(&L.down, false, false));
      if (L.gate.tag != MINQ_F32 && L.gate.tag == L.up.tag) {
        MINQ_TRY(prepare_map(&L.gate, true, true));
        MINQ_TRY(prepare_map(&L.up, true, true));
      }
    }
  }
  uint64_t nf = 0;
  MINQ_TRY(get_vec(m, "model.norm.weight", true, &m->final_norm, &nf));
  check_vec(m, m->final_norm, nf, H, "model.norm");
  if (m->pending.count("lm_head.weight")) {
    MINQ_TRY(get_linear(m, "lm_head.weight", &m->lm_head));
  } else {  // tied embeddings (model.rs:561-565), aliased instead of cloned
    m->lm_head.tag = MINQ_F32;
    m->lm_head.rows = emb->shape[0];
    m->lm_head.cols = emb->shape[1];
    m->lm_head.ptr = emb->ptr;
    m->lm_head.nbytes = emb->nbytes;
  }
  check_linear(m, m->lm_head, m->lm_head.rows, H, "lm_head");
  if (m->shape_error.empty() && m->lm_head.rows < c.vocab_size)
    m->shape_error = "lm_head has fewer rows than vocab_size";
  m->weight_bytes += m->lm_head.nbytes;
  if (m->lm_head.tag == MINQ_F32 && (H % 4 != 0) && m->shape_error.empty())
    m->shape_error = "hidden_size must be a multiple of 4 for the f32 lm_head kernel";
  if (m->shape_error.empty() && m->lm_head.tag != MINQ_F32) {
    DevLinear& lm = m->lm_head;
    if (lm.cols % 128 == 0 && (uintptr_t)lm.ptr % 16 == 0) {
      const QmvPlan t = plan_qmatvec_tma(lm.tag, false, c.vocab_size, (int)lm.cols, true);
      MINQ_TRY(encode_qmatvec_map(lm.ptr, c.vocab_size, (int)lm.cols, lm.tag, t.nr, &lm.tm));
      lm.tm_ok = true;
    }
  }

  // RoPE tables.
  std::vector<float> cs, sn;
  build_rope_tables(hd, c.max_seq_len, c.rope_theta, &cs, &sn);
  void *pc, *ps;
  MINQ_TRY(dmalloc(m, &pc, cs.size() * 4));
  MINQ_TRY(dmalloc(m, &ps, sn.size() * 4));
  m->rope_cos = static_cast<float*>(pc);
  m->rope_sin = static_cast<float*>(ps);
  MINQ_CUDA_TRY(cudaMemcpy(pc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  MINQ_CUDA_TRY(cudaMemcpy(ps, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));

  // Activation scratch.
  const uint64_t V = m->lm_head.rows;
  const uint64_t big = std::max<uint64_t>({qd + 2 * kvd, I, H, V, 1});
  void* p;
  auto alloc_f = [&](float** dst, uint64_t n) -> minq_status {
    MINQ_TRY(dmalloc(m, &p, n * 4));
    *dst = static_cast<float*>(p);
    return MINQ_OK;
  };
  MINQ_TRY(alloc_f(&m->x, H));
  MINQ_TRY(alloc_f(&m->xn, H));
  MINQ_TRY(alloc_f(&m->qkv, qd + 2 * kvd));
  MINQ_TRY(alloc_f(&m->q_rot, qd));
  MINQ_TRY(alloc_f(&m->att, qd));
  MINQ_TRY(alloc_f(&m->hbuf, I));
  MINQ_TRY(alloc_f(&m->gbuf, I));
  MINQ_TRY(alloc_f(&m->ubuf, I));
  MINQ_TRY(alloc_f(&m->tmp, big));
  MINQ_TRY(alloc_f(&m->logits, V));
  m->argmax_cap = argmax_parts_capacity();
  MINQ_TRY(dmalloc(m, &p, m->argmax_cap * sizeof(unsigned long long)));
  m->argmax_part = static_cast<unsigned long long*>(p);
  MINQ_TRY(dmalloc(m, &p, 16));
  m->d_tok = static_cast<uint32_t*>(p);
  MINQ_CUDA_TRY(cudaMemsetAsync(m->d_tok, 0, 16, m->stream));
  m->d_tokens_cap = 4096;
  MINQ_TRY(dmalloc(m, &p, m->d_tokens_cap * 4));
  m->d_tokens = static_cast<uint32_t*>(p);
  if (!device_status_word()) return fail(MINQ_ERR_CUDA, "cannot allocate the device status word");
  m->nh_l = (int)c.n_heads;
  m->nkv_l = (int)c.n_kv_heads;
  m->I_l = c.intermediate_size;
  if (m->shape_error.empty()) MINQ_TRY(setup_megakernel(m));
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  m->finished = true;
  return MINQ_OK;
}

namespace {

// y = L x (+ bias) (+ residual), optionally with RMSNorm(x; norm_w) applied
// first. Quantized weights use the fused matvec; dense f32 weights use the
// f32 matvec then an elementwise epilogue.
minq_status linear(minq_model* m, const DevLinear& l, const float* x, const float* norm_w,
                   const float* bias, const float* residual, float* y) {
  const float eps = m->cfg.rms_norm_eps;
  if (l.tag != MINQ_F32)
    return launch_qmatvec(l.tag, l.ptr, nullptr, l.rows, (int)l.cols, x, norm_w, eps, bias,
                          residual, y, m->stream, norm_w ? nullptr : map_of(l));
  const bool epi = bias || residual;
  float* dst = epi ? m->tmp : y;
  if (l.cols % 4 != 0) return fail(MINQ_ERR_SHAPE, "f32 matvec needs cols % 4 == 0");
  MINQ_TRY(launch_f32_matvec(static_cast<const float*>(l.ptr), l.rows, (int)l.cols, x, norm_w,
                             eps, dst, nullptr, nullptr, m->stream));
  if (epi) MINQ_TRY(launch_epilogue(m->tmp, bias, residual, y, l.rows, m->stream));
  return MINQ_OK;
}

}  // namespace

// x = sum over the tensor-parallel ranks of x (in place, on the model
// stream); `site` numbers the all-reduce within the token (2 per layer).
static minq_status tp_allreduce_x(minq_model* m, int site) {
  if (m->tpar.on) return launch_tp_allreduce(m->tpar, m->x, site, m->stream);
  const NcclApi& nc = nccl_api();
  ncclResult_t r = nc.AllReduce(m->x, m->x, m->cfg.hidden_size, ncclFloat, ncclSum,
                                static_cast<ncclComm_t>(m->tp_comm), m->stream);
  r = nccl_settle(static_cast<ncclComm_t>(m->tp_comm), r,
                  std::chrono::steady_clock::now() + std::chrono::seconds(30));
  if (r != ncclSuccess) return fail(MINQ_ERR_NCCL, std::string("ncclAllReduce: ") + nc.GetErrorString(r));
  return MINQ_OK;
}

// model.rs:273-318 for one token. The token id is read from `d_tok`. In
// graph mode the position comes from c->d_pos (device) and the attention
// grid is sized for the cache capacity; otherwise `pos` is used. Logits (and
// their argmax into d_argmax) only when `want_logits`.
minq_status forward_token(minq_model* m, minq_cache* c, const uint32_t* d_tok, size_t pos,
                          bool want_logits, float* d_logits, uint32_t* d_argmax, bool graph) {
  const minq_config& cfg = m->cfg;
  const int H = (int)cfg.hidden_size, hd = (int)cfg.head_dim, nh = m->nh_l, nkv = m->nkv_l;
  const uint64_t qd = (uint64_t)nh * hd, kvd = (uint64_t)nkv * hd, I = m->I_l;
  const float eps = cfg.rms_norm_eps;
  cudaStream_t s = m->stream;
  // tensor parallel: o_proj and down_proj give partial sums of x's update;
  // rank 0 adds the residual, then an all-reduce sums the ranks into x
  const bool tp = m->tp_world > 1;
  const float* res = tp && m->tp_rank != 0 ? nullptr : m->x;
  const size_t seq_stride = (size_t)nkv * c->max_seq * hd, head_stride = c->max_seq * hd,
               pos_stride = hd;
  const size_t layer_elems = c->batch * seq_stride;
  const int* dpos = graph ? c->d_pos : nullptr;
  MINQ_TRY(launch_embed(m->embed, d_tok, cfg.vocab_size, H, m->x, s));
  for (uint64_t li = 0; li < cfg.n_layers; ++li) {
    const DevLayer& L = m->layers[li];
    // attention sub-layer: q|k|v = W (rmsnorm(x)) + bias
    if (L.qkv.tag >= 0) {
      MINQ_TRY(launch_qmatvec(L.qkv.tag, L.qkv.ptr, nullptr, L.qkv.rows, H, m->x, L.attn_norm,
                              eps, L.bias_qkv, nullptr, m->qkv, s, map_of(L.qkv)));
    } else {
      MINQ_TRY(launch_rmsnorm(m->x, L.attn_norm, eps, H, m->xn, s));
      MINQ_TRY(linear(m, L.q, m->xn, nullptr, L.q_bias, nullptr, m->qkv));
      MINQ_TRY(linear(m, L.k, m->xn, nullptr, L.k_bias, nullptr, m->qkv + qd));
      MINQ_TRY(linear(m, L.v, m->xn, nullptr, L.v_bias, nullptr, m->qkv + qd + kvd));
    }
    float* kc = c->k + li * layer_elems;
    float* vc = c->v + li * layer_elems;
    MINQ_TRY(launch_rope_append(m->qkv, m->qkv + qd, m->qkv + qd + kvd, 0, 0, L.q_norm,
                                L.k_norm, eps, m->rope_cos, m->rope_sin, 1, nh, nkv, hd,
                                (int)pos, m->q_rot, kc, vc, seq_stride, head_stride, pos_stride,
                                s, dpos));
    MINQ_TRY(launch_attention(m->q_rot, kc, vc, 1, nh, nkv, hd, (int)pos + 1, seq_stride,
                              head_stride, pos_stride, m->att, c->ws, c->ws_bytes, s, dpos,
                              (int)c->max_seq));
    MINQ_TRY(linear(m, L.o, m->att, nullptr, nullptr, res, m->x));  // x += o
    if (tp) MINQ_TRY(tp_allreduce_x(m, (int)(2 * li)));
    // MLP sub-layer: h = silu(gate(rmsnorm(x))) * up(rmsnorm(x)); x += down(h)
    if (L.gate.tag != MINQ_F32 && L.gate.tag == L.up.tag) {
      MINQ_TRY(launch_qmatvec(L.gate.tag, L.gate.ptr, L.up.ptr, I, H, m->x, L.ffn_norm, eps,
                              nullptr, nullptr, m->hbuf, s, map_of(L.gate), map_of(L.up)));
    } else {
      MINQ_TRY(launch_rmsnorm(m->x, L.ffn_norm, eps, H, m->xn, s));
      MINQ_TRY(linear(m, L.gate, m->xn, nullptr, nullptr, nullptr, m->gbuf));
      MINQ_TRY(linear(m, L.up, m->xn, nullptr, nullptr, nullptr, m->ubuf));
      MINQ_TRY(launch_swiglu(m->gbuf, m->ubuf, m->hbuf, I, s));
    }
    MINQ_TRY(linear(m, L.down, m->hbuf, nullptr, nullptr, res, m->x));  // x += down
    if (tp) MINQ_TRY(tp_allreduce_x(m, (int)(2 * li + 1)));
  }
  if (tp && m->tpar.on) MINQ_TRY(launch_tp_ar_advance(m->tpar, s));
  if (want_logits) {
    const uint64_t V = cfg.vocab_size;
    if (m->lm_head.tag == MINQ_F32) {
      int nparts = m->argmax_cap;
      MINQ_TRY(launch_f32_matvec(static_cast<const float*>(m->lm_head.ptr), V, H, m->x,
                                 m->final_norm, eps, d_logits, m->argmax_part, &nparts, s));
      MINQ_TRY(launch_argmax_final(m->argmax_part, nparts, d_argmax, s));
    } else {
      MINQ_TRY(launch_qmatvec(m->lm_head.tag, m->lm_head.ptr, nullptr, V, H, m->x,
                              m->final_norm, eps, nullptr, nullptr, d_logits, s,
                              map_of(m->lm_head)));
      MINQ_TRY(launch_argmax(d_logits, V, m->argmax_part, m->argmax_cap, d_argmax, s));
    }
  }
  if (graph) MINQ_TRY(launch_advance_pos(c->d_pos, 1, s));
  return MINQ_OK;
}

// model.rs:273-318 for the `batch` sequences of cache c, one token each
// (c->btok), all at position c->len: the same steps as forward_token with
// every projection a batched matvec (weights read once for the batch).
static minq_status forward_batch_step(minq_model* m, minq_cache* c, bool want_logits) {
  const minq_config& cfg = m->cfg;
  const int H = (int)cfg.hidden_size, hd = (int)cfg.head_dim, nh = (int)cfg.n_heads,
            nkv = (int)cfg.n_kv_heads, B = (int)c->batch;
  const uint64_t qd = (uint64_t)nh * hd, kvd = (uint64_t)nkv * hd, I = cfg.intermediate_size;
  const uint64_t qkv_rows = qd + 2 * kvd, V = cfg.vocab_size;
  const float eps = cfg.rms_norm_eps;
  const int pos = (int)c->len;
  cudaStream_t s = m->stream;
  const size_t seq_stride = (size_t)nkv * c->max_seq * hd, head_stride = c->max_seq * hd;
  const size_t layer_elems = c->batch * seq_stride;
  MINQ_TRY(launch_embed_batch(m->embed, c->btok, V, H, B, c->bx, s));
  for (uint64_t li = 0; li < cfg.n_layers; ++li) {
    const DevLayer& L = m->layers[li];
    MINQ_TRY(launch_qmatmul(L.qkv.tag, L.qkv.ptr, nullptr, qkv_rows, H, B, c->bx, H, L.attn_norm,
                            eps, c->bxn, c->bxn_floats, L.bias_qkv, nullptr, c->bqkv, qkv_rows,
                            c->bpart, c->bpart_floats, s));
    float* kc = c->k + li * layer_elems;
    float* vc = c->v + li * layer_elems;
    MINQ_TRY(launch_rope_append(c->bqkv, c->bqkv + qd, c->bqkv + qd + kvd, qkv_rows, qkv_rows,
                                L.q_norm, L.k_norm, eps, m->rope_cos, m->rope_sin, c->batch, nh,
                                nkv, hd, pos, c->bq, kc, vc, seq_stride, head_stride, hd, s));
    MINQ_TRY(launch_attention(c->bq, kc, vc, c->batch, nh, nkv, hd, pos + 1, seq_stride,
                              head_stride, hd, c->batt, c->ws, c->ws_bytes, s));
    MINQ_TRY(launch_qmatmul(L.o.tag, L.o.ptr, nullptr, H, (int)qd, B, c->batt, qd, nullptr, eps,
                            c->bxn, c->bxn_floats, nullptr, c->bx, c->bx, H, c->bpart,
                            c->bpart_floats, s));  // x += o
    MINQ_TRY(launch_qmatmul(L.gate.tag, L.gate.ptr, L.up.ptr, I, H, B, c->bx, H, L.ffn_norm, eps,
                            c->bxn, c->bxn_floats, nullptr, nullptr, c->bh, I, c->bpart,
                            c->bpart_floats, s));  // silu(gate) * up
    MINQ_TRY(launch_qmatmul(L.down.tag, L.down.ptr, nullptr, H, (int)I, B, c->bh, I, nullptr, eps,
                            c->bxn, c->bxn_floats, nullptr, c->bx, c->bx, H, c->bpart,
                            c->bpart_floats, s));  // x += down
  }
  if (want_logits) {
    MINQ_TRY(launch_qmatmul(m->lm_head.tag, m->lm_head.ptr, nullptr, V, H, B, c->bx, H,
                            m->final_norm, eps, c->bxn, c->bxn_floats, nullptr, nullptr, c->blog, V,
                            c->bpart, c->bpart_floats, s));
    // the lm_head's slice partials are consumed: bpart takes the argmax parts
    MINQ_TRY(launch_argmax_rows(c->blog, V, B, c->barg,
                                reinterpret_cast<unsigned long long*>(c->bpart), s));
  }
  return MINQ_OK;
}

// The batched step's activations (first use) and its shape requirements.
static minq_status batch_ready(minq_model* m, minq_cache* c) {
  const minq_config& cfg = m->cfg;
  if (m->tp_world > 1) return fail(MINQ_ERR_ARG, "the batched step runs on one GPU");
  if (c->batch > (size_t)kQmmMaxB)
    return fail(MINQ_ERR_ARG, "minq_forward_batch takes at most 64 sequences per cache");
  if (cfg.hidden_size % 32 || cfg.intermediate_size % 32 || (cfg.n_heads * cfg.head_dim) % 32)
    return fail(MINQ_ERR_SHAPE, "the batched step needs 32-column blocks");
  for (const DevLayer& L : m->layers)
    if (L.qkv.tag < 0 || L.gate.tag == MINQ_F32 || L.gate.tag != L.up.tag)
      return fail(MINQ_ERR_SHAPE,
                  "the batched step needs quantized q|k|v and gate/up projections of one dtype");
  if (c->bx) return MINQ_OK;
  const size_t B = c->batch, H = cfg.hidden_size, I = cfg.intermediate_size,
               qd = cfg.n_heads * cfg.head_dim, kvd = cfg.n_kv_heads * cfg.head_dim,
               V = cfg.vocab_size;
  auto alloc = [&](void** dst, size_t bytes) -> minq_status {  // owned by the cache
    MINQ_CUDA_TRY(cudaMalloc(dst, bytes ? bytes : 16));
    return MINQ_OK;
  };
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bx), B * H * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bqkv), B * (qd + 2 * kvd) * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bq), B * qd * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->batt), B * qd * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bh), B * I * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->blog), B * V * 4));
  c->bxn_floats = B * std::max({H, qd, I});
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bxn), c->bxn_floats * 4));
  c->bpart_floats = 4 * B * std::max({H, qd + 2 * kvd, I});
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->bpart), c->bpart_floats * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->btok), B * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->barg), B * 4));
  return MINQ_OK;
}

// Chunked prompt prefill: kPrefillChunk prompt tokens of a batch-1 cache per
// pass, the projections as batched matvecs over the chunk's tokens (tensor
// cores from two tokens on), RoPE / cache append at consecutive positions,
// and attention with causal per-token histories (token i of a chunk at
// position p0 + i attends over p0 + i + 1 positions). The same steps as
// forward_token (model.rs:273-318) for each token, without the lm_head: the
// prompt's last token runs as a decode step, which also gives the logits.
constexpr int kPrefillChunk = kQmmMaxB;

// Whether the model takes chunked prefill (the batched step's shape rules,
// one GPU), and its activations on first use. MINQ_CHUNKED_PREFILL=0 turns
// chunked prompts off (use_env); the full-sequence sweep ignores it.
static minq_status prefill_ready(minq_model* m, minq_cache* c, bool* ok, bool use_env = true,
                                  bool any_batch = false) {
  *ok = false;
  const minq_config& cfg = m->cfg;
  const char* env = std::getenv("MINQ_CHUNKED_PREFILL");
  if (use_env && env && env[0] == '0') return MINQ_OK;
  if (m->tp_world > 1 || (c->batch != 1 && !any_batch)) return MINQ_OK;
  if (cfg.hidden_size % 32 || cfg.intermediate_size % 32 || (cfg.n_heads * cfg.head_dim) % 32)
    return MINQ_OK;
  for (const DevLayer& L : m->layers)
    if (L.qkv.tag < 0 || L.gate.tag == MINQ_F32 || L.gate.tag != L.up.tag) return MINQ_OK;
  *ok = true;
  if (c->px) return MINQ_OK;
  const size_t B = kPrefillChunk, H = cfg.hidden_size, I = cfg.intermediate_size,
               qd = cfg.n_heads * cfg.head_dim, kvd = cfg.n_kv_heads * cfg.head_dim;
  auto alloc = [&](void** dst, size_t bytes) -> minq_status {  // owned by the cache
    MINQ_CUDA_TRY(cudaMalloc(dst, bytes ? bytes : 16));
    return MINQ_OK;
  };
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->px), B * H * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->pqkv), B * (qd + 2 * kvd) * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->pq), B * qd * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->patt), B * qd * 4));
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->ph), B * I * 4));
  c->pxn_floats = B * std::max({H, qd, I});
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->pxn), c->pxn_floats * 4));
  c->ppart_floats = 4 * B * std::max({H, qd + 2 * kvd, I});
  MINQ_TRY(alloc(reinterpret_cast<void**>(&c->ppart), c->ppart_floats * 4));
  // the attention's split partials for any chunk size at any history
  size_t ws = 0;
  for (size_t t = 1; t <= B; ++t)
    ws = std::max(ws, attn_workspace_need(t, (int)cfg.n_heads, (int)cfg.n_kv_heads,
                                          (int)cfg.head_dim, (int)c->max_seq, true));
  ws = std::max(ws, prefill_attention_workspace((int)B, (int)cfg.n_heads, (int)cfg.n_kv_heads,
                                                (int)cfg.head_dim));
  c->pws_bytes = ws + 256;
  MINQ_TRY(alloc(&c->pws, c->pws_bytes));
  return MINQ_OK;
}

// T <= kPrefillChunk tokens (device ids) at positions c->len .. c->len + T - 1.
static minq_status forward_chunk(minq_model* m, minq_cache* c, const uint32_t* d_toks, int T,
                                 size_t seq = 0) {
  const minq_config& cfg = m->cfg;
  const int H = (int)cfg.hidden_size, hd = (int)cfg.head_dim, nh = (int)cfg.n_heads,
            nkv = (int)cfg.n_kv_heads;
  const uint64_t qd = (uint64_t)nh * hd, kvd = (uint64_t)nkv * hd, I = cfg.intermediate_size;
  const uint64_t qkv_rows = qd + 2 * kvd, V = cfg.vocab_size;
  const float eps = cfg.rms_norm_eps;
  const int p0 = (int)c->len;
  cudaStream_t s = m->stream;
  // sequence `seq` of the cache ([layer][batch][kv head][max_seq][hd])
  const size_t seq_elems = (size_t)nkv * c->max_seq * hd, layer_elems = c->batch * seq_elems,
               head_stride = c->max_seq * hd;
  // causal chunk attention: the tensor-core kernel for head_dim 64 / 128
  // (MINQ_FLASH_PREFILL=0: the split-KV decode kernel, one entry per token)
  static const bool flash_env = [] {
    const char* e = std::getenv("MINQ_FLASH_PREFILL");
    return !(e && e[0] == '0');
  }();
  const bool flash = flash_env && prefill_attention_supported(nh, nkv, hd) &&
                     (uintptr_t)c->k % 16 == 0 && (uintptr_t)c->v % 16 == 0;
  MINQ_TRY(launch_embed_batch(m->embed, d_toks, V, H, T, c->px, s));
  for (uint64_t li = 0; li < cfg.n_layers; ++li) {
    const DevLayer& L = m->layers[li];
    MINQ_TRY(launch_qmatmul(L.qkv.tag, L.qkv.ptr, nullptr, qkv_rows, H, T, c->px, H, L.attn_norm,
                            eps, c->pxn, c->pxn_floats, L.bias_qkv, nullptr, c->pqkv, qkv_rows,
                            c->ppart, c->ppart_floats, s));
    float* kc = c->k + li * layer_elems + seq * seq_elems;
    float* vc = c->v + li * layer_elems + seq * seq_elems;
    // token i: rotated at position p0 + i and appended there (one sequence:
    // sequence stride 0), then attends over p0 + i + 1 positions
    MINQ_TRY(launch_rope_append(c->pqkv, c->pqkv + qd, c->pqkv + qd + kvd, qkv_rows, qkv_rows,
                                L.q_norm, L.k_norm, eps, m->rope_cos, m->rope_sin, (size_t)T, nh,
                                nkv, hd, p0, c->pq, kc, vc, 0, head_stride, hd, s, nullptr, 1));
    if (flash)  // every token of the chunk at once on the tensor cores
      MINQ_TRY(launch_prefill_attention(c->pq, kc, vc, head_stride, p0, T, nh, nkv, hd, c->patt,
                                        c->pws, c->pws_bytes, s));
    else
      MINQ_TRY(launch_attention(c->pq, kc, vc, (size_t)T, nh, nkv, hd, p0 + 1, 0, head_stride,
                                hd, c->patt, c->pws, c->pws_bytes, s, nullptr, 0, true, 1));
    MINQ_TRY(launch_qmatmul(L.o.tag, L.o.ptr, nullptr, H, (int)qd, T, c->patt, qd, nullptr, eps,
                            c->pxn, c->pxn_floats, nullptr, c->px, c->px, H, c->ppart,
                            c->ppart_floats, s));  // x += o
    MINQ_TRY(launch_qmatmul(L.gate.tag, L.gate.ptr, L.up.ptr, I, H, T, c->px, H, L.ffn_norm, eps,
                            c->pxn, c->pxn_floats, nullptr, nullptr, c->ph, I, c->ppart,
                            c->ppart_floats, s));  // silu(gate) * up
    MINQ_TRY(launch_qmatmul(L.down.tag, L.down.ptr, nullptr, H, (int)I, T, c->ph, I, nullptr, eps,
                            c->pxn, c->pxn_floats, nullptr, c->px, c->px, H, c->ppart,
                            c->ppart_floats, s));  // x += down
  }
  c->len += (size_t)T;
  c->d_pos_valid = false;
  return MINQ_OK;
}

// Capture one decode step (with or without logits) of cache `c` as a graph.
static minq_status capture_step(minq_model* m, minq_cache* c, bool logits, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  MINQ_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  minq_status st = forward_token(m, c, m->d_tok, 0, logits, m->logits, m->d_tok, true);
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (st != MINQ_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
  return MINQ_OK;
}

static minq_status sync_dpos(minq_cache* c) {
  if (c->d_pos_valid) return MINQ_OK;
  const int v = (int)c->len;
  MINQ_CUDA_TRY(cudaMemcpyAsync(c->d_pos, &v, sizeof(int), cudaMemcpyHostToDevice, c->m->stream));
  MINQ_CUDA_TRY(cudaStreamSynchronize(c->m->stream));
  c->d_pos_valid = true;
  return MINQ_OK;
}

// One decode step of a batch-1 cache as the megakernel.
static minq_status run_megakernel(minq_model* m, minq_cache* c, bool logits) {
  const minq_config& cfg = m->cfg;
  auto& k = m->mk;
  MkParams p{};
  p.layers = k.layers;
  p.n_layers = (int)cfg.n_layers;
  p.qkv = k.qkv;
  p.o = k.o;
  p.gu = k.gu;
  p.down = k.down;
  p.H = (int)cfg.hidden_size;
  p.I = (int)m->I_l;
  p.nh = m->nh_l;
  p.nkv = m->nkv_l;
  p.hd = (int)cfg.head_dim;
  p.G = p.nh / p.nkv;
  p.qd = p.nh * p.hd;
  p.kvd = p.nkv * p.hd;
  p.nsplit = k.nsplit;
  p.vocab = (int)cfg.vocab_size;
  p.eps = cfg.rms_norm_eps;
  p.scale = 1.0f / sqrtf((float)cfg.head_dim);
  p.embed = m->embed;
  p.lm_head = static_cast<const float*>(m->lm_head.ptr);
  p.final_norm = m->final_norm;
  p.rope_cos = m->rope_cos;
  p.rope_sin = m->rope_sin;
  p.kc = c->k;
  p.vc = c->v;
  p.cache_layer_stride = (size_t)p.nkv * c->max_seq * p.hd;
  p.max_seq = (int)c->max_seq;
  p.x = m->x;
  p.qkv_out = m->qkv;
  p.att = m->att;
  p.h = m->hbuf;
  p.logits = m->logits;
  p.part = k.part;
  p.head_ctr = k.head_ctr;
  p.head_base = k.head_base;
  p.argmax_part = k.argmax_part;
  p.d_tok = m->d_tok;
  p.d_pos = c->d_pos;
  p.bar_ctr = k.bar;
  p.bar_base = k.bar + 1;
  p.status = device_status_word();
  p.abort_flag = k.abort_flag;
  p.want_logits = logits ? 1 : 0;
  p.scratch_bytes = k.scratch;
  p.tp_world = m->tp_world;
  p.tp_rank = m->tp_rank;
  if (m->tp_world > 1) {  // every rank's exchange slots, mapped at minq_tp_init
    p.xr_dst = reinterpret_cast<uint2* const*>(m->tpar.peer_recv);
    p.xr_local = reinterpret_cast<const uint2*>(m->tpar.recv);
    p.xr_epoch = reinterpret_cast<unsigned*>(m->tpar.ctr);
  } else {
    p.xr_dst = k.xr_dst;
    p.xr_local = k.xr;
    p.xr_epoch = k.xr_epoch;
  }
  return launch_decode_mk(p, k.dtype, k.grid, k.smem, m->stream);
}

// Clear the megakernel's barrier / merge state after a device-side timeout.
static minq_status reset_megakernel(minq_model* m) {
  auto& k = m->mk;
  if (!k.ok) return MINQ_OK;
  const size_t nkv = m->cfg.n_kv_heads;
  MINQ_CUDA_TRY(cudaMemsetAsync(k.bar, 0, nkv * 4 + 4 + 2 * 8 + (size_t)k.grid * 8 + 64,
                                m->stream));
  if (m->tp_world == 1 && k.xr)  // pairs of an aborted launch must not match the next epoch
    MINQ_CUDA_TRY(cudaMemsetAsync(k.xr, 0, 2 * m->cfg.n_layers * m->cfg.hidden_size * sizeof(uint2) + 256,
                                  m->stream));
  return MINQ_OK;
}

// Run one step for the token already in m->d_tok (megakernel, graph replay or
// eager).
static minq_status run_step(minq_model* m, minq_cache* c, bool logits) {
  if (m->mk.ok && c->batch == 1) {
    MINQ_TRY(sync_dpos(c));
    MINQ_TRY(run_megakernel(m, c, logits));
    c->len += 1;
    return MINQ_OK;
  }
  if (m->use_graphs) {
    MINQ_TRY(sync_dpos(c));
    cudaGraphExec_t& g = c->step[logits ? 1 : 0];
    if (!g) MINQ_TRY(capture_step(m, c, logits, &g));
    MINQ_CUDA_TRY(cudaGraphLaunch(g, m->stream));
  } else {
    c->d_pos_valid = false;
    MINQ_TRY(forward_token(m, c, m->d_tok, c->len, logits, m->logits, m->d_tok, false));
  }
  c->len += 1;
  return MINQ_OK;
}

}  // namespace minq

using namespace minq;

// ---------------------------------------------------------------------------
// C ABI: model

extern "C" {

minq_status minq_model_new(const minq_config* cfg, minq_model** out) {
  if (!cfg || !out) return fail(MINQ_ERR_ARG, "null argument");
  int dev_count = 0;
  cudaError_t e = cudaGetDeviceCount(&dev_count);
  if (e != cudaSuccess || dev_count == 0)
    return fail(MINQ_ERR_CUDA, "no CUDA device available (the CUDA path has no CPU fallback)");
  minq_model* m = new minq_model();
  m->cfg = *cfg;
  cudaGetDevice(&m->device);
  const char* g = std::getenv("MINQ_GRAPHS");
  m->use_graphs = !(g && g[0] == '0');
  e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete m;
    return cuda_fail(e, "cudaStreamCreate");
  }
  *out = m;
  return MINQ_OK;
}

// The record checks of minq_model_add_tensor (format.rs:212-249): a known
// storage tag, 2-D block-aligned quantized shapes, data length equal to the
// shape-derived byte count.
static minq_status check_record(const char* name, minq_dtype tag, size_t ndim,
                                const uint64_t* shape, size_t nbytes) {
  if (tag != MINQ_F32 && tag != MINQ_Q8_0 && tag != MINQ_Q4_0)
    return fail(MINQ_ERR_FORMAT, std::string("tensor `") + name + "`: unknown storage tag " +
                                     std::to_string((int)tag));
  uint64_t numel = 1;
  for (size_t i = 0; i < ndim; ++i) numel *= shape[i];
  uint64_t expected;
  if (tag == MINQ_F32) {
    expected = numel * 4;
  } else {
    if (ndim != 2)
      return fail(MINQ_ERR_FORMAT, std::string("quantized tensor `") + name + "` must be 2-D");
    if (shape[1] % 32 != 0)
      return fail(MINQ_ERR_FORMAT,
                  std::string("quantized tensor `") + name + "`: cols not block-aligned");
    expected = shape[0] * (shape[1] / 32) * (uint64_t)block_bytes(tag);
  }
  if (expected != nbytes)
    return fail(MINQ_ERR_FORMAT, std::string("tensor `") + name + "`: data length " +
                                     std::to_string(nbytes) + " != shape-derived " +
                                     std::to_string(expected));
  return MINQ_OK;
}

// Records the device tensor under its name; the last record of a name wins,
// like the reference's HashMap (its earlier buffer stays in m->allocs).
static void put_tensor(minq_model* m, const char* name, DevTensor t) {
  auto it = m->pending.find(name);
  if (it != m->pending.end()) it->second = t;
  else m->pending.emplace(name, t);
}

minq_status minq_model_add_tensor(minq_model* m, const char* name, minq_dtype tag, size_t ndim,
                                  const uint64_t* shape, const void* data, size_t nbytes,
                                  int data_on_device) {
  if (!m || !name || (ndim && !shape) || (nbytes && !data))
    return fail(MINQ_ERR_ARG, "null argument");
  if (m->finished) return fail(MINQ_ERR_MODEL, "model already finished");
  MINQ_TRY(check_record(name, tag, ndim, shape, nbytes));
  DevTensor t;
  t.tag = tag;
  t.shape.assign(shape, shape + ndim);
  t.nbytes = nbytes;
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  void* p;
  MINQ_TRY(dmalloc(m, &p, nbytes));
  t.ptr = p;
  MINQ_CUDA_TRY(cudaMemcpy(p, data, nbytes,
                           data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  put_tensor(m, name, t);
  return MINQ_OK;
}

// Host-to-device upload of mapped file bytes through two pinned staging
// buffers on a copy stream: while one buffer's cudaMemcpyAsync runs, host
// threads fill the other from the mapping (the first touch of a mapped page
// reads it from the file). One cudaMemcpyAsync per chunk.
namespace {
struct PinnedUpload {
  cudaStream_t s = nullptr;
  unsigned char* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool busy[2] = {false, false};
  size_t chunk = 0;
  int next = 0;
  unsigned threads = 1;

  minq_status init() {
    chunk = size_t(64) << 20;
    if (const char* e = std::getenv("MINQ_LOAD_CHUNK_BYTES"))
      chunk = std::max<size_t>(4096, std::strtoull(e, nullptr, 10));
    threads = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    MINQ_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
      MINQ_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&buf[i]), chunk, cudaHostAllocDefault));
      MINQ_CUDA_TRY(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
    }
    return MINQ_OK;
  }
  ~PinnedUpload() {
    if (s) cudaStreamSynchronize(s);
    for (int i = 0; i < 2; ++i) {
      if (ev[i]) cudaEventDestroy(ev[i]);
      if (buf[i]) cudaFreeHost(buf[i]);
    }
    if (s) cudaStreamDestroy(s);
  }
  void fill(unsigned char* dst, const unsigned char* src, size_t n) {
    const unsigned t = n >= (size_t(8) << 20) ? threads : 1u;
    if (t == 1) {
      std::memcpy(dst, src, n);
      return;
    }
    std::vector<std::thread> pool;
    const size_t part = (n + t - 1) / t;
    for (unsigned i = 0; i < t; ++i) {
      const size_t a = i * part, b = std::min(n, a + part);
      if (a < b) pool.emplace_back([=] { std::memcpy(dst + a, src + a, b - a); });
    }
    for (auto& th : pool) th.join();
  }
  minq_status copy(void* dev, const unsigned char* src, size_t n) {
    for (size_t off = 0; off < n; off += chunk) {
      const size_t len = std::min(chunk, n - off);
      const int b = next;
      next ^= 1;
      if (busy[b]) MINQ_CUDA_TRY(cudaEventSynchronize(ev[b]));
      fill(buf[b], src + off, len);
      MINQ_CUDA_TRY(cudaMemcpyAsync(static_cast<unsigned char*>(dev) + off, buf[b], len,
                                    cudaMemcpyHostToDevice, s));
      MINQ_CUDA_TRY(cudaEventRecord(ev[b], s));
      busy[b] = true;
    }
    return MINQ_OK;
  }
  minq_status finish() {
    MINQ_CUDA_TRY(cudaStreamSynchronize(s));
    return MINQ_OK;
  }
};
}  // namespace

static minq_status upload_records(minq_model* m, const MinqMapping& map,
                                  const std::vector<MinqRecord>& recs) {
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  PinnedUpload up;
  MINQ_TRY(up.init());
  for (const MinqRecord& r : recs) {
    MINQ_TRY(check_record(r.name.c_str(), (minq_dtype)r.tag, r.shape.size(), r.shape.data(),
                          r.nbytes));
    DevTensor t;
    t.tag = (minq_dtype)r.tag;
    t.shape = r.shape;
    t.nbytes = r.nbytes;
    void* p;
    MINQ_TRY(dmalloc(m, &p, r.nbytes));
    t.ptr = p;
    MINQ_TRY(up.copy(p, map.base + r.offset, r.nbytes));
    put_tensor(m, r.name.c_str(), t);
  }
  return up.finish();
}

minq_status minq_model_finish(minq_model* m) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  if (m->finished) return MINQ_OK;
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  return model_finish(m);
}

minq_status minq_model_load(const char* path, minq_model** out) {
  if (!path || !out) return fail(MINQ_ERR_ARG, "null argument");
  minq_config cfg{};
  std::vector<MinqRecord> recs;
  MinqMapping map;
  std::string err;
  minq_status st = index_minq_file(path, &cfg, &recs, &map, &err);
  if (st != MINQ_OK) return fail(st, err);
  minq_model* m = nullptr;
  MINQ_TRY(minq_model_new(&cfg, &m));
  st = upload_records(m, map, recs);
  if (st == MINQ_OK) st = minq_model_finish(m);
  if (st != MINQ_OK) {
    std::string msg = minq_last_error();
    minq_model_free(m);
    return fail(st, msg);
  }
  *out = m;
  return MINQ_OK;
}

minq_status minq_model_config(const minq_model* m, minq_config* out) {
  if (!m || !out) return fail(MINQ_ERR_ARG, "null argument");
  *out = m->cfg;
  return MINQ_OK;
}

minq_status minq_model_weight_bytes(const minq_model* m, uint64_t* out) {
  if (!m || !out) return fail(MINQ_ERR_ARG, "null argument");
  *out = m->weight_bytes;
  return MINQ_OK;
}

minq_status minq_model_set_graphs(minq_model* m, int enabled) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  m->use_graphs = enabled != 0;
  return MINQ_OK;
}

void* minq_model_stream(minq_model* m) { return m ? (void*)m->stream : nullptr; }

minq_status minq_debug_inject_timeout(minq_model* m, int what) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  auto& k = m->mk;
  if (!k.ok) return fail(MINQ_ERR_ARG, "the decode megakernel is not in use for this model");
  if (what != 0 && what != 1) return fail(MINQ_ERR_ARG, "what: 0 (head counters) or 1 (grid barrier)");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  if (what == 0) {  // the next launch's per-head merge targets lie 2^30 splits ahead
    unsigned v = 0;
    MINQ_CUDA_TRY(cudaMemcpy(&v, k.head_base, 4, cudaMemcpyDeviceToHost));
    v += 1u << 30;
    MINQ_CUDA_TRY(cudaMemcpy(k.head_base, &v, 4, cudaMemcpyHostToDevice));
  } else {          // the next launch's grid-barrier targets lie 2^40 arrivals ahead
    unsigned long long v = 0;
    MINQ_CUDA_TRY(cudaMemcpy(&v, k.bar + 1, 8, cudaMemcpyDeviceToHost));
    v += 1ull << 40;
    MINQ_CUDA_TRY(cudaMemcpy(k.bar + 1, &v, 8, cudaMemcpyHostToDevice));
  }
  return MINQ_OK;
}

void minq_model_free(minq_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (minq_cache* c : m->caches) {  // caches still open: release them, keep the handles
    cache_release_device(c);
    c->m = nullptr;
  }
  m->caches.clear();
  minq::tp_ar_release(&m->tpar);
  if (m->tp_comm) nccl_api().CommDestroy(static_cast<ncclComm_t>(m->tp_comm));
  for (void* p : m->allocs) cudaFree(p);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

// ---------------------------------------------------------------------------
// C ABI: tensor parallelism

minq_status minq_tp_unique_id(void* id_out) {
  if (!id_out) return fail(MINQ_ERR_ARG, "null argument");
  const NcclApi& nc = nccl_api();
  if (!nc.ok) return fail(MINQ_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = nc.GetUniqueId(&id);
  if (r != ncclSuccess) return fail(MINQ_ERR_NCCL, std::string("ncclGetUniqueId: ") + nc.GetErrorString(r));
  std::memcpy(id_out, &id, sizeof(id));
  return MINQ_OK;
}

namespace {

// Rows [r0, r1) of a quantized linear as a new device matrix.
minq_status tp_rows(minq_model* m, DevLinear* l, uint64_t r0, uint64_t r1) {
  const size_t rb = l->nbytes / l->rows;
  void* p;
  MINQ_TRY(dmalloc(m, &p, (r1 - r0) * rb));
  MINQ_CUDA_TRY(cudaMemcpyAsync(p, static_cast<const char*>(l->ptr) + r0 * rb, (r1 - r0) * rb,
                                cudaMemcpyDeviceToDevice, m->stream));
  l->ptr = p;
  l->rows = r1 - r0;
  l->nbytes = (r1 - r0) * rb;
  l->tm_ok = false;
  return MINQ_OK;
}

// Columns [c0, c1) (block aligned) of a quantized linear as a new matrix.
minq_status tp_cols(minq_model* m, DevLinear* l, uint64_t c0, uint64_t c1) {
  const size_t rb = l->nbytes / l->rows, bb = rb / (l->cols / 32);
  const size_t nrb = (c1 - c0) / 32 * bb;
  void* p;
  MINQ_TRY(dmalloc(m, &p, l->rows * nrb));
  MINQ_CUDA_TRY(cudaMemcpy2DAsync(p, nrb, static_cast<const char*>(l->ptr) + c0 / 32 * bb, rb, nrb,
                                  l->rows, cudaMemcpyDeviceToDevice, m->stream));
  l->ptr = p;
  l->cols = c1 - c0;
  l->nbytes = l->rows * nrb;
  l->tm_ok = false;
  return MINQ_OK;
}

// Rows [r0, r1) of q, k and v of the fused matrix (and its bias) as a new
// fused matrix.
minq_status tp_qkv(minq_model* m, DevLayer* L, uint64_t q0, uint64_t q1, uint64_t k0, uint64_t k1,
                   uint64_t v0, uint64_t v1) {
  DevLinear& l = L->qkv;
  const size_t rb = l.nbytes / l.rows, n = (q1 - q0) + (k1 - k0) + (v1 - v0);
  void* p;
  MINQ_TRY(dmalloc(m, &p, n * rb));
  char* d = static_cast<char*>(p);
  const char* src = static_cast<const char*>(l.ptr);
  size_t at = 0;
  for (auto [a, b] : {std::pair<uint64_t, uint64_t>{q0, q1}, {k0, k1}, {v0, v1}}) {
    MINQ_CUDA_TRY(cudaMemcpyAsync(d + at * rb, src + a * rb, (b - a) * rb,
                                  cudaMemcpyDeviceToDevice, m->stream));
    at += b - a;
  }
  if (L->bias_qkv) {
    void* bp;
    MINQ_TRY(dmalloc(m, &bp, n * 4));
    float* bd = static_cast<float*>(bp);
    at = 0;
    for (auto [a, b] : {std::pair<uint64_t, uint64_t>{q0, q1}, {k0, k1}, {v0, v1}}) {
      MINQ_CUDA_TRY(cudaMemcpyAsync(bd + at, L->bias_qkv + a, (b - a) * 4,
                                    cudaMemcpyDeviceToDevice, m->stream));
      at += b - a;
    }
    L->bias_qkv = bd;
  }
  l.ptr = p;
  l.rows = n;
  l.nbytes = n * rb;
  l.tm_ok = false;
  return MINQ_OK;
}

}  // namespace

minq_status minq_tp_init(minq_model* m, int rank, int world, const void* unique_id) {
  if (!m || !unique_id) return fail(MINQ_ERR_ARG, "null argument");
  if (!m->finished) return fail(MINQ_ERR_MODEL, "model not finished");
  if (world < 1 || rank < 0 || rank >= world) return fail(MINQ_ERR_ARG, "bad rank / world");
  if (m->tp_world > 1) return fail(MINQ_ERR_ARG, "tensor parallelism already set up");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  const minq_config& c = m->cfg;
  const uint64_t hd = c.head_dim, nh = c.n_heads, nkv = c.n_kv_heads, I = c.intermediate_size;
  if (nh % world || nkv % world || I % (32ull * world) || (nh / world * hd) % 32)
    return fail(MINQ_ERR_SHAPE, "heads and intermediate rows must split evenly over the ranks "
                                "in 32-column blocks");
  for (const DevLayer& L : m->layers)
    if (L.qkv.tag < 0 || L.o.tag == MINQ_F32 || L.down.tag == MINQ_F32 || L.gate.tag == MINQ_F32 ||
        L.up.tag == MINQ_F32)
      return fail(MINQ_ERR_SHAPE, "tensor parallelism needs quantized projections");
  const NcclApi& nc = nccl_api();
  if (!nc.ok) return fail(MINQ_ERR_NCCL, "libnccl.so.2 could not be loaded");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  // the ranks meet under a host deadline (MINQ_TP_INIT_TIMEOUT_S, default
  // 120 s): a non-blocking communicator is polled and aborted when a rank
  // never joins, so the call returns MINQ_ERR_NCCL instead of blocking
  const char* tenv = std::getenv("MINQ_TP_INIT_TIMEOUT_S");
  const double tmo = tenv && std::atof(tenv) > 0 ? std::atof(tenv) : 120.0;
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::milliseconds((long long)(tmo * 1000.0));
  ncclResult_t r;
  if (nc.nonblocking) {
    ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
    ncfg.blocking = 0;
    r = nc.CommInitRankConfig(&comm, world, id, rank, &ncfg);
    if (r == ncclInProgress || r == ncclSuccess) {
      r = nccl_settle(comm, ncclInProgress, deadline);
      if (r == ncclInProgress)
        return fail(MINQ_ERR_NCCL, "ncclCommInitRank: the ranks did not all join within " +
                                       std::to_string(tmo) + " s (communicator aborted)");
    }
  } else {
    r = nc.CommInitRank(&comm, world, id, rank);
  }
  if (r != ncclSuccess) {
    if (comm && nc.CommAbort) nc.CommAbort(comm);
    return fail(MINQ_ERR_NCCL, std::string("ncclCommInitRank: ") + nc.GetErrorString(r));
  }
  // this rank's heads and intermediate rows (q/k/v rows by head, gate/up
  // rows, o_proj / down_proj columns)
  const uint64_t nhl = nh / world, nkvl = nkv / world, Il = I / world, qd = nh * hd, kvd = nkv * hd;
  const uint64_t q0 = rank * nhl * hd, k0 = rank * nkvl * hd, i0 = rank * Il;
  for (DevLayer& L : m->layers) {
    MINQ_TRY(tp_qkv(m, &L, q0, q0 + nhl * hd, qd + k0, qd + k0 + nkvl * hd, qd + kvd + k0,
                    qd + kvd + k0 + nkvl * hd));
    MINQ_TRY(tp_cols(m, &L.o, q0, q0 + nhl * hd));
    MINQ_TRY(tp_rows(m, &L.gate, i0, i0 + Il));
    MINQ_TRY(tp_rows(m, &L.up, i0, i0 + Il));
    MINQ_TRY(tp_cols(m, &L.down, i0, i0 + Il));
    MINQ_TRY(prepare_map(&L.qkv, false, true));
    MINQ_TRY(prepare_map(&L.o, false, false));
    MINQ_TRY(prepare_map(&L.down, false, false));
    if (L.gate.tag == L.up.tag) {
      MINQ_TRY(prepare_map(&L.gate, true, true));
      MINQ_TRY(prepare_map(&L.up, true, true));
    }
  }
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  if (tp_ar_wanted())
    MINQ_TRY(tp_ar_setup(&m->tpar, rank, world, (int)c.hidden_size, (int)(2 * c.n_layers), comm,
                         m->stream));
  m->tp_comm = comm;
  m->tp_rank = rank;
  m->tp_world = world;
  m->nh_l = (int)nhl;
  m->nkv_l = (int)nkvl;
  m->I_l = Il;
  // the decode megakernel runs the rank's slices when the peer all-reduce
  // slots are mapped and the shapes fit it; otherwise the per-op step runs
  // (graph-captured with its all-reduces)
  m->mk.ok = false;
  if (m->tpar.on) MINQ_TRY(setup_megakernel(m));
  return MINQ_OK;
}

// ---------------------------------------------------------------------------
// C ABI: cache

minq_status minq_cache_new(minq_model* m, size_t batch, size_t max_seq, minq_cache** out) {
  if (!m || !out) return fail(MINQ_ERR_ARG, "null argument");
  if (!m->finished) return fail(MINQ_ERR_MODEL, "model not finished");
  if (batch == 0) return fail(MINQ_ERR_ARG, "batch must be >= 1");
  if (max_seq == 0 || max_seq > m->cfg.max_seq_len) max_seq = m->cfg.max_seq_len;
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  minq_cache* c = new minq_cache();
  c->m = m;
  c->batch = batch;
  c->max_seq = max_seq;
  const size_t per_layer = batch * (size_t)m->nkv_l * max_seq * m->cfg.head_dim;
  const size_t bytes = m->cfg.n_layers * per_layer * sizeof(float);
  cudaError_t e = cudaMalloc(&c->k, bytes ? bytes : 16);
  if (e == cudaSuccess) e = cudaMalloc(&c->v, bytes ? bytes : 16);
  c->ws_bytes = attn_workspace_bytes(batch, (size_t)m->nh_l, max_seq, m->cfg.head_dim);
  if (e == cudaSuccess) e = cudaMalloc(&c->ws, c->ws_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_pos, 16);
  if (e != cudaSuccess) {
    cudaFree(c->k);
    cudaFree(c->v);
    cudaFree(c->ws);
    cudaFree(c->d_pos);
    delete c;
    return cuda_fail(e, "cudaMalloc(kv cache)");
  }
  m->caches.insert(c);
  *out = c;
  return MINQ_OK;
}

minq_status minq_cache_reset(minq_cache* c) {
  if (!c) return fail(MINQ_ERR_ARG, "null cache");
  c->len = 0;
  c->d_pos_valid = false;
  return MINQ_OK;
}

minq_status minq_cache_len(const minq_cache* c, size_t* out) {
  if (!c || !out) return fail(MINQ_ERR_ARG, "null argument");
  *out = c->len;
  return MINQ_OK;
}

minq_status minq_cache_set_len(minq_cache* c, size_t len) {
  if (!c) return fail(MINQ_ERR_ARG, "null cache");
  if (len > c->max_seq) return fail(MINQ_ERR_MODEL, "length exceeds cache capacity");
  c->len = len;
  c->d_pos_valid = false;
  return MINQ_OK;
}

static minq_status cache_copy(const minq_cache* c, size_t layer, size_t start, size_t n,
                              float* host_k, float* host_v, bool to_device,
                              cudaMemcpyKind in_kind = cudaMemcpyHostToDevice) {
  const minq_config& cfg = c->m->cfg;
  if (layer >= cfg.n_layers) return fail(MINQ_ERR_SHAPE, "layer out of range");
  if (start + n > c->max_seq) return fail(MINQ_ERR_SHAPE, "positions exceed cache capacity");
  if (n == 0) return MINQ_OK;
  const size_t hd = cfg.head_dim, nkv = (size_t)c->m->nkv_l;
  const size_t per_layer = c->batch * nkv * c->max_seq * hd;
  MINQ_CUDA_TRY(cudaSetDevice(c->m->device));
  for (int which = 0; which < 2; ++which) {
    float* dev = (which ? c->v : c->k) + layer * per_layer;
    float* host = which ? host_v : host_k;
    if (!host) continue;
    for (size_t h = 0; h < nkv; ++h) {
      float* d = dev + h * c->max_seq * hd + start * hd;
      float* hp = host + h * hd;
      if (to_device)
        MINQ_CUDA_TRY(cudaMemcpy2D(d, hd * 4, hp, nkv * hd * 4, hd * 4, n, in_kind));
      else
        MINQ_CUDA_TRY(cudaMemcpy2D(hp, nkv * hd * 4, d, hd * 4, hd * 4, n,
                                   cudaMemcpyDeviceToHost));
    }
  }
  return MINQ_OK;
}

minq_status minq_cache_write(minq_cache* c, size_t layer, size_t start, size_t n, const float* k,
                             const float* v) {
  if (!c) return fail(MINQ_ERR_ARG, "null cache");
  MINQ_CUDA_TRY(cudaStreamSynchronize(c->m->stream));
  return cache_copy(c, layer, start, n, const_cast<float*>(k), const_cast<float*>(v), true);
}

minq_status minq_cache_write_device(minq_cache* c, size_t layer, size_t start, size_t n,
                                    const float* d_k, const float* d_v) {
  if (!c) return fail(MINQ_ERR_ARG, "null cache");
  MINQ_CUDA_TRY(cudaStreamSynchronize(c->m->stream));
  return cache_copy(c, layer, start, n, const_cast<float*>(d_k), const_cast<float*>(d_v), true,
                    cudaMemcpyDeviceToDevice);
}

minq_status minq_cache_read(const minq_cache* c, size_t layer, size_t start, size_t n, float* k,
                            float* v) {
  if (!c) return fail(MINQ_ERR_ARG, "null cache");
  MINQ_CUDA_TRY(cudaStreamSynchronize(c->m->stream));
  return cache_copy(c, layer, start, n, k, v, false);
}

// A cache outlived by its model (freed first, e.g. by a garbage collector
// finalising both in any order) had its device memory released with the
// model; only the handle remains.
void minq_cache_free(minq_cache* c) {
  if (!c) return;
  if (c->m) {
    cudaSetDevice(c->m->device);
    cudaStreamSynchronize(c->m->stream);
    cache_release_device(c);
    c->m->caches.erase(c);
  }
  delete c;
}

// ---------------------------------------------------------------------------
// C ABI: forward / generate

// Common checks, then one step per token; token i comes from host h_tokens
// or device d_tokens. Results land in m->logits / m->d_tok.
static minq_status forward_impl(minq_model* m, minq_cache* c, const uint32_t* h_tokens,
                                const uint32_t* d_tokens, size_t n) {
  if (!m || !c) return fail(MINQ_ERR_ARG, "null argument");
  if (c->m != m) return fail(MINQ_ERR_ARG, "cache belongs to another model");
  if (n == 0) return fail(MINQ_ERR_MODEL, "empty token sequence");  // model.rs:255-257
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  if (c->batch != 1) return fail(MINQ_ERR_ARG, "minq_forward drives a batch-1 cache");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  const uint32_t* toks = d_tokens;
  if (h_tokens) {
    MINQ_TRY(reserve_tokens(m, n));
    MINQ_CUDA_TRY(cudaMemcpyAsync(m->d_tokens, h_tokens, n * 4, cudaMemcpyHostToDevice,
                                  m->stream));
    toks = m->d_tokens;
  }
  size_t i = 0;
  bool chunked = false;
  if (n >= 2 && c->len + n <= m->cfg.max_seq_len && c->len + n <= c->max_seq)
    MINQ_TRY(prefill_ready(m, c, &chunked));
  // a prompt with an out-of-range token goes token by token, so the valid
  // tokens before it are processed and the error comes at that token
  if (chunked && h_tokens)
    for (size_t j = 0; j < n; ++j) chunked = chunked && h_tokens[j] < m->cfg.vocab_size;
  if (chunked) {
    // every token but the last in chunks; the last one below gives the logits
    for (; i + 1 < n; i += kPrefillChunk) {
      const int T = (int)std::min<size_t>(kPrefillChunk, n - 1 - i);
      MINQ_TRY(forward_chunk(m, c, toks + i, T));
    }
    i = n - 1;
  }
  for (; i < n; ++i) {
    if (c->len >= m->cfg.max_seq_len)  // model.rs:260-265
      return fail(MINQ_ERR_MODEL,
                  "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq_len) + ")");
    if (c->len >= c->max_seq)
      return fail(MINQ_ERR_MODEL,
                  "sequence exceeds the cache capacity (" + std::to_string(c->max_seq) + ")");
    if (h_tokens && h_tokens[i] >= m->cfg.vocab_size)  // Tensor::row (tensor.rs:73-78)
      return fail(MINQ_ERR_SHAPE, "row index " + std::to_string(h_tokens[i]) +
                                      " out of bounds for " + std::to_string(m->cfg.vocab_size) +
                                      " rows");
    MINQ_CUDA_TRY(cudaMemcpyAsync(m->d_tok, toks + i, 4, cudaMemcpyDeviceToDevice, m->stream));
    MINQ_TRY(run_step(m, c, i + 1 == n));
  }
  return MINQ_OK;
}

minq_status minq_forward_device(minq_model* m, minq_cache* c, const uint32_t* d_tokens,
                                size_t n, float* d_logits, uint32_t* d_argmax) {
  if (!d_tokens) return fail(MINQ_ERR_ARG, "null tokens");
  MINQ_TRY(forward_impl(m, c, nullptr, d_tokens, n));
  if (d_logits && d_logits != m->logits)
    MINQ_CUDA_TRY(cudaMemcpyAsync(d_logits, m->logits, m->cfg.vocab_size * 4,
                                  cudaMemcpyDeviceToDevice, m->stream));
  if (d_argmax && d_argmax != m->d_tok)
    MINQ_CUDA_TRY(cudaMemcpyAsync(d_argmax, m->d_tok, 4, cudaMemcpyDeviceToDevice, m->stream));
  return MINQ_OK;
}

minq_status minq_decode_steps(minq_model* m, minq_cache* c, size_t n_steps,
                              uint32_t* d_tokens_out) {
  if (!m || !c) return fail(MINQ_ERR_ARG, "null argument");
  if (c->m != m) return fail(MINQ_ERR_ARG, "cache belongs to another model");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  if (c->batch != 1) return fail(MINQ_ERR_ARG, "minq_decode_steps drives a batch-1 cache");
  if (c->len == 0) return fail(MINQ_ERR_MODEL, "decode continuation needs a prefilled cache");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  for (size_t i = 0; i < n_steps; ++i) {
    if (c->len >= m->cfg.max_seq_len)
      return fail(MINQ_ERR_MODEL,
                  "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq_len) + ")");
    if (c->len >= c->max_seq)
      return fail(MINQ_ERR_MODEL,
                  "sequence exceeds the cache capacity (" + std::to_string(c->max_seq) + ")");
    MINQ_TRY(run_step(m, c, true));
    if (d_tokens_out)
      MINQ_CUDA_TRY(cudaMemcpyAsync(d_tokens_out + i, m->d_tok, 4, cudaMemcpyDeviceToDevice,
                                    m->stream));
  }
  return MINQ_OK;
}

minq_status minq_forward_batch(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                               float* logits_out, uint32_t* argmax_out) {
  if (!m || !c) return fail(MINQ_ERR_ARG, "null argument");
  if (c->m != m) return fail(MINQ_ERR_ARG, "cache belongs to another model");
  if (n == 0 || !tokens) return fail(MINQ_ERR_MODEL, "empty token sequence");
  if (n != c->batch) return fail(MINQ_ERR_ARG, "one token per sequence of the cache");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  if (c->len >= m->cfg.max_seq_len)  // model.rs:260-265
    return fail(MINQ_ERR_MODEL,
                "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq_len) + ")");
  if (c->len >= c->max_seq)
    return fail(MINQ_ERR_MODEL,
                "sequence exceeds the cache capacity (" + std::to_string(c->max_seq) + ")");
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= m->cfg.vocab_size)  // Tensor::row (tensor.rs:73-78)
      return fail(MINQ_ERR_SHAPE, "row index " + std::to_string(tokens[i]) +
                                      " out of bounds for " + std::to_string(m->cfg.vocab_size) +
                                      " rows");
  MINQ_TRY(batch_ready(m, c));
  MINQ_CUDA_TRY(cudaMemcpyAsync(c->btok, tokens, n * 4, cudaMemcpyHostToDevice, m->stream));
  const bool want = logits_out || argmax_out;
  MINQ_TRY(forward_batch_step(m, c, want));
  c->len += 1;
  c->d_pos_valid = false;
  if (logits_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(logits_out, c->blog, n * m->cfg.vocab_size * 4,
                                  cudaMemcpyDeviceToHost, m->stream));
  if (argmax_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(argmax_out, c->barg, n * 4, cudaMemcpyDeviceToHost, m->stream));
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return take_device_status();
}

minq_status minq_forward_batch_device(minq_model* m, minq_cache* c, size_t n_steps,
                                      uint32_t* d_tokens_out) {
  if (!m || !c) return fail(MINQ_ERR_ARG, "null argument");
  if (c->m != m) return fail(MINQ_ERR_ARG, "cache belongs to another model");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  if (c->len == 0 || !c->bx) return fail(MINQ_ERR_MODEL, "decode continuation needs a prefilled cache");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  for (size_t i = 0; i < n_steps; ++i) {
    if (c->len >= m->cfg.max_seq_len || c->len >= c->max_seq)
      return fail(MINQ_ERR_MODEL, "sequence exceeds the cache capacity");
    MINQ_CUDA_TRY(cudaMemcpyAsync(c->btok, c->barg, c->batch * 4, cudaMemcpyDeviceToDevice,
                                  m->stream));
    MINQ_TRY(forward_batch_step(m, c, true));
    c->len += 1;
    if (d_tokens_out)
      MINQ_CUDA_TRY(cudaMemcpyAsync(d_tokens_out + i * c->batch, c->barg, c->batch * 4,
                                    cudaMemcpyDeviceToDevice, m->stream));
  }
  c->d_pos_valid = false;
  return MINQ_OK;
}

minq_status minq_forward(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                         float* logits_out, uint32_t* argmax_out) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  if (n && !tokens) return fail(MINQ_ERR_ARG, "null tokens");
  minq_status st = forward_impl(m, c, tokens, nullptr, n);
  if (st != MINQ_OK) {
    cudaStreamSynchronize(m->stream);
    return st;
  }
  if (logits_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(logits_out, m->logits, m->cfg.vocab_size * 4,
                                  cudaMemcpyDeviceToHost, m->stream));
  if (argmax_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(argmax_out, m->d_tok, 4, cudaMemcpyDeviceToHost, m->stream));
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  const minq_status ds = take_device_status();
  if (ds != MINQ_OK) reset_megakernel(m);
  return ds;
}

minq_status minq_generate(minq_model* m, const uint32_t* prompt, size_t n_prompt,
                          size_t max_tokens, const uint32_t* stop_tokens, size_t n_stop,
                          minq_token_cb on_token, void* user, uint32_t* tokens_out,
                          minq_gen_stats* stats) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  if (n_prompt == 0) return fail(MINQ_ERR_MODEL, "empty prompt");  // engine.rs:58-60
  minq_cache* c = nullptr;
  MINQ_TRY(minq_cache_new(m, 1, 0, &c));
  using clk = std::chrono::steady_clock;
  minq_gen_stats st{};
  st.prompt_tokens = n_prompt;
  uint32_t tok = 0;
  auto t0 = clk::now();
  minq_status rc = minq_forward(m, c, prompt, n_prompt, nullptr, &tok);
  st.prefill_secs = std::chrono::duration<double>(clk::now() - t0).count();
  auto t1 = clk::now();
  for (size_t i = 0; rc == MINQ_OK && i < max_tokens; ++i) {
    if (tokens_out) tokens_out[i] = tok;
    if (on_token && on_token(tok, user) != 0) {
      rc = fail(MINQ_ERR_MODEL, "on_token callback aborted generation");
      break;
    }
    st.gen_tokens += 1;
    bool stop = false;
    for (size_t k = 0; k < n_stop; ++k) stop |= stop_tokens[k] == tok;
    if (stop) break;
    uint32_t next;
    rc = minq_forward(m, c, &tok, 1, nullptr, &next);
    tok = next;
  }
  st.decode_secs = std::chrono::duration<double>(clk::now() - t1).count();
  minq_cache_free(c);
  if (stats) *stats = st;
  return rc;
}

minq_status minq_generate_sampled(minq_model* m, minq_sampler* smp, const uint32_t* prompt,
                                  size_t n_prompt, size_t max_tokens,
                                  const uint32_t* stop_tokens, size_t n_stop,
                                  minq_token_cb on_token, void* user, uint32_t* tokens_out,
                                  minq_gen_stats* stats) {
  if (!m || !smp) return fail(MINQ_ERR_ARG, "null argument");
  if (n_prompt == 0) return fail(MINQ_ERR_MODEL, "empty prompt");  // engine.rs:58-60
  if (sampler_device(smp) != m->device)
    return fail(MINQ_ERR_ARG, "the sampler lives on another device than the model");
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  minq_cache* c = nullptr;
  MINQ_TRY(minq_cache_new(m, 1, 0, &c));
  uint32_t* d_tok = nullptr;
  if (cudaMalloc(&d_tok, 16) != cudaSuccess) {
    minq_cache_free(c);
    return fail(MINQ_ERR_CUDA, "cudaMalloc(token)");
  }
  using clk = std::chrono::steady_clock;
  minq_gen_stats st{};
  st.prompt_tokens = n_prompt;
  auto t0 = clk::now();
  minq_status rc = minq_forward(m, c, prompt, n_prompt, nullptr, nullptr);
  st.prefill_secs = std::chrono::duration<double>(clk::now() - t0).count();
  auto t1 = clk::now();
  for (size_t i = 0; rc == MINQ_OK && i < max_tokens; ++i) {
    // Sampler::sample on the step's logits (engine.rs:72), on the device
    rc = minq_sampler_sample_device(smp, m->logits, m->cfg.vocab_size, d_tok, m->stream);
    uint32_t tok = 0;
    if (rc == MINQ_OK) {
      cudaError_t e = cudaMemcpyAsync(&tok, d_tok, 4, cudaMemcpyDeviceToHost, m->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
      if (e != cudaSuccess) rc = cuda_fail(e, "sampled token");
    }
    if (rc != MINQ_OK) break;
    if (tokens_out) tokens_out[i] = tok;
    if (on_token && on_token(tok, user) != 0) {
      rc = fail(MINQ_ERR_MODEL, "on_token callback aborted generation");
      break;
    }
    st.gen_tokens += 1;
    bool stop = false;
    for (size_t k = 0; k < n_stop; ++k) stop |= stop_tokens[k] == tok;
    if (stop) break;
    rc = forward_impl(m, c, nullptr, d_tok, 1);  // logits of the next step
  }
  if (rc == MINQ_OK) rc = take_device_status();
  st.decode_secs = std::chrono::duration<double>(clk::now() - t1).count();
  cudaFree(d_tok);
  minq_cache_free(c);
  if (stats) *stats = st;
  return rc;
}

// ---------------------------------------------------------------------------
// C ABI: full-sequence states and perplexity (model.rs:337-424, ppl.rs:44-103)

// Token ids to the device (m->d_tokens), after the common checks.
static minq_status upload_tokens(minq_model* m, const uint32_t* h, size_t n) {
  MINQ_TRY(reserve_tokens(m, n));
  MINQ_CUDA_TRY(cudaMemcpyAsync(m->d_tokens, h, n * 4, cudaMemcpyHostToDevice, m->stream));
  return MINQ_OK;
}

static minq_status check_rows(const minq_model* m, const uint32_t* t, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (t[i] >= m->cfg.vocab_size)  // Tensor::row (tensor.rs:73-78)
      return fail(MINQ_ERR_SHAPE, "row index " + std::to_string(t[i]) + " out of bounds for " +
                                      std::to_string(m->cfg.vocab_size) + " rows");
  return MINQ_OK;
}

minq_status minq_prefill_batch(minq_model* m, minq_cache* c, const uint32_t* tokens, size_t n,
                               float* logits_out, uint32_t* argmax_out) {
  if (!m || !c) return fail(MINQ_ERR_ARG, "null argument");
  if (c->m != m) return fail(MINQ_ERR_ARG, "cache belongs to another model");
  if (n == 0 || !tokens) return fail(MINQ_ERR_MODEL, "empty token sequence");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  const size_t B = c->batch;
  if (c->len + n > m->cfg.max_seq_len)  // model.rs:260-265
    return fail(MINQ_ERR_MODEL,
                "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq_len) + ")");
  if (c->len + n > c->max_seq)
    return fail(MINQ_ERR_MODEL,
                "sequence exceeds the cache capacity (" + std::to_string(c->max_seq) + ")");
  MINQ_TRY(check_rows(m, tokens, B * n));
  MINQ_TRY(batch_ready(m, c));
  bool chunked = false;
  MINQ_TRY(prefill_ready(m, c, &chunked, true, true));
  const size_t p0 = c->len;
  std::vector<uint32_t> col(B);
  if (chunked && n > 1) {
    // every sequence's prompt but its last token, in chunks of 64 tokens at
    // the common positions p0 .. p0 + n - 2 of that sequence's cache
    MINQ_TRY(upload_tokens(m, tokens, B * n));
    for (size_t b = 0; b < B; ++b) {
      c->len = p0;
      for (size_t i = 0; i + 1 < n; i += kPrefillChunk) {
        const int T = (int)std::min<size_t>(kPrefillChunk, n - 1 - i);
        minq_status st = forward_chunk(m, c, m->d_tokens + b * n + i, T, b);
        if (st != MINQ_OK) {
          c->len = p0;
          return st;
        }
      }
    }
    c->len = p0 + n - 1;
    c->d_pos_valid = false;
  } else {
    for (size_t i = 0; i + 1 < n; ++i) {  // one batched step per prompt position
      for (size_t b = 0; b < B; ++b) col[b] = tokens[b * n + i];
      MINQ_CUDA_TRY(cudaMemcpyAsync(c->btok, col.data(), B * 4, cudaMemcpyHostToDevice, m->stream));
      MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
      MINQ_TRY(forward_batch_step(m, c, false));
      c->len += 1;
      c->d_pos_valid = false;
    }
  }
  // the last prompt token of every sequence as one batched step (logits)
  for (size_t b = 0; b < B; ++b) col[b] = tokens[b * n + n - 1];
  MINQ_CUDA_TRY(cudaMemcpyAsync(c->btok, col.data(), B * 4, cudaMemcpyHostToDevice, m->stream));
  const bool want = logits_out || argmax_out;
  MINQ_TRY(forward_batch_step(m, c, want));
  c->len += 1;
  c->d_pos_valid = false;
  if (logits_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(logits_out, c->blog, B * m->cfg.vocab_size * 4,
                                  cudaMemcpyDeviceToHost, m->stream));
  if (argmax_out)
    MINQ_CUDA_TRY(cudaMemcpyAsync(argmax_out, c->barg, B * 4, cudaMemcpyDeviceToHost, m->stream));
  MINQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return take_device_status();
}

// A batch-1 scratch cache of max_seq positions with the chunk buffers (and,
// for scoring, [chunk][vocab] logits and [chunk] nll).
static minq_status sweep_cache(minq_model* m, size_t max_seq, bool scoring, minq_cache** out) {
  minq_cache* c = nullptr;
  MINQ_TRY(minq_cache_new(m, 1, max_seq, &c));
  bool ok = false;
  minq_status st = prefill_ready(m, c, &ok, false);
  if (st == MINQ_OK && !ok)
    st = fail(MINQ_ERR_SHAPE,
              "the full-sequence sweep needs one GPU, quantized q|k|v and gate/up projections "
              "and 32-column blocks");
  if (st == MINQ_OK && scoring) {
    const size_t V = m->cfg.vocab_size;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->plog), kPrefillChunk * V * 4);
    // one f64 nll per scored position of a window (read once per window)
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->pnll), max_seq * 8);
    if (e != cudaSuccess) st = cuda_fail(e, "cudaMalloc(perplexity buffers)");
  }
  if (st != MINQ_OK) {
    minq_cache_free(c);
    return st;
  }
  *out = c;
  return MINQ_OK;
}

minq_status minq_forward_full_states(minq_model* m, const uint32_t* tokens, size_t n,
                                     float* states_out) {
  if (!m) return fail(MINQ_ERR_ARG, "null model");
  if (!m->finished) return fail(MINQ_ERR_MODEL, "model not finished");
  if (n == 0) return fail(MINQ_ERR_MODEL, "empty token sequence");  // model.rs:326-328
  if (!tokens) return fail(MINQ_ERR_ARG, "null tokens");
  if (n > m->cfg.max_seq_len)                                         // model.rs:331-336
    return fail(MINQ_ERR_MODEL,
                "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq_len) + ")");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  MINQ_TRY(check_rows(m, tokens, n));
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  MINQ_TRY(upload_tokens(m, tokens, n));
  minq_cache* c = nullptr;
  MINQ_TRY(sweep_cache(m, n, false, &c));
  const size_t H = m->cfg.hidden_size;
  minq_status st = MINQ_OK;
  for (size_t i = 0; st == MINQ_OK && i < n; i += kPrefillChunk) {
    const int T = (int)std::min<size_t>(kPrefillChunk, n - i);
    st = forward_chunk(m, c, m->d_tokens + i, T);
    if (st == MINQ_OK && states_out) {
      const cudaError_t e = cudaMemcpyAsync(states_out + i * H, c->px, (size_t)T * H * 4,
                                            cudaMemcpyDeviceToHost, m->stream);
      if (e != cudaSuccess) st = cuda_fail(e, "cudaMemcpyAsync(states)");
    }
  }
  if (st == MINQ_OK) {
    const cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) st = cuda_fail(e, "cudaStreamSynchronize");
  }
  if (st == MINQ_OK) st = take_device_status();
  minq_cache_free(c);
  return st;
}

minq_status minq_eval_ppl(minq_model* m, const uint32_t* tokens, size_t n, size_t context,
                          minq_ppl_window_cb on_window, void* user, minq_ppl_result* out) {
  if (!m || !tokens || !out) return fail(MINQ_ERR_ARG, "null argument");
  if (!m->finished) return fail(MINQ_ERR_MODEL, "model not finished");
  if (n < 3)  // ppl.rs:51-68
    return fail(MINQ_ERR_MODEL, "need at least 3 tokens to score, got " + std::to_string(n));
  if (context < 3)
    return fail(MINQ_ERR_MODEL, "context must be >= 3, got " + std::to_string(context));
  if (context > m->cfg.max_seq_len)
    return fail(MINQ_ERR_MODEL, "context " + std::to_string(context) + " exceeds max_seq_len (" +
                                    std::to_string(m->cfg.max_seq_len) + ")");
  if (!m->shape_error.empty()) return fail(MINQ_ERR_SHAPE, m->shape_error);
  MINQ_CUDA_TRY(cudaSetDevice(m->device));
  MINQ_TRY(upload_tokens(m, tokens, n));
  minq_cache* c = nullptr;
  MINQ_TRY(sweep_cache(m, context, true, &c));
  const size_t H = m->cfg.hidden_size, V = m->cfg.vocab_size;
  const size_t n_windows = (n + context - 1) / context;
  cudaStream_t s = m->stream;
  double nll_sum = 0.0;
  std::vector<double> part(context);
  size_t count = 0;
  minq_status st = MINQ_OK;
  for (size_t w0 = 0, wi = 0; st == MINQ_OK && w0 < n; w0 += context, ++wi) {
    const size_t len = std::min(context, n - w0);
    // the reference's sweep of this window fails at an out-of-range row
    // after the earlier windows have been reported
    if ((st = check_rows(m, tokens + w0, len)) != MINQ_OK) break;
    c->len = 0;
    c->d_pos_valid = false;
    // positions 0 .. len - 2: the last one predicts nothing (ppl.rs:75-82);
    // the chunks' nll values stay on the device until the window ends, so
    // the host enqueues the next chunk while the GPU runs this one
    size_t wn = 0;
    for (size_t i = 0; st == MINQ_OK && i + 1 < len; i += kPrefillChunk) {
      const int T = (int)std::min<size_t>(kPrefillChunk, len - 1 - i);
      if ((st = forward_chunk(m, c, m->d_tokens + w0 + i, T)) != MINQ_OK) break;
      const int r0 = i == 0 ? 1 : 0;  // position 0 has no left context
      const int R = T - r0;
      if (R <= 0) continue;
      // final RMSNorm fused into the lm_head over the chunk's scored rows
      st = launch_qmatmul(m->lm_head.tag, m->lm_head.ptr, nullptr, V, (int)H, R, c->px + r0 * H,
                          H, m->final_norm, m->cfg.rms_norm_eps, c->pxn, c->pxn_floats, nullptr,
                          nullptr, c->plog, V, c->ppart, c->ppart_floats, s);
      if (st == MINQ_OK)
        st = launch_nll_rows(c->plog, V, R, m->d_tokens + w0 + i + r0 + 1, c->pnll + wn, s);
      if (st != MINQ_OK) break;
      wn += (size_t)R;
    }
    if (st == MINQ_OK && wn) {
      cudaError_t e = cudaMemcpyAsync(part.data(), c->pnll, wn * 8, cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) {
        st = cuda_fail(e, "perplexity window");
        break;
      }
      for (size_t r = 0; r < wn; ++r) nll_sum += part[r];  // position order, as ppl.rs:81
      count += wn;
    }
    if (st == MINQ_OK && on_window)
      on_window(wi + 1, n_windows, count ? std::exp(nll_sum / (double)count) : NAN, user);
  }
  if (st == MINQ_OK) st = take_device_status();
  minq_cache_free(c);
  if (st != MINQ_OK) return st;
  if (count == 0)  // ppl.rs:93-97
    return fail(MINQ_ERR_MODEL, "no scorable positions (sequence too short for context)");
  out->total_tokens = n;
  out->scored_positions = count;
  out->mean_nll = nll_sum / (double)count;
  out->ppl = std::exp(out->mean_nll);
  return MINQ_OK;
}

}  // extern "C"
