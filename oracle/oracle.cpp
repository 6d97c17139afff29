// CPU ORACLE — TEST INFRASTRUCTURE ONLY.
//
// A C++17 restatement of minq's CPU forward path (kn1g78/minq, Rust), used as
// the parity reference for the CUDA library and as the timed CPU baseline. Only the
// test suite, `__graft_entry__.smoke()` and `bench.py`'s CPU legs load it; the
// product library (minq_b200/libminq_cuda.so) never links or calls it.
//
// Every function follows the reference's f32 operation order (no FMA
// contraction outside the explicit AVX2 intrinsics, which mirror the
// reference's own `_mm256_fmadd_ps` calls). Citations are `path:line` inside
// the reference project.
//
// Parity pins: the reference ships no golden vectors, so the oracle is pinned
// by the reference's own known-answer and equivalence tests (quantize.rs:420-
// 513, tensor.rs:251-307, model.rs:747-940, sampler.rs:261-301, format.rs:311-
// 434), restated in tests/test_oracle_pins.py, plus golden fixtures produced
// by an independent numpy restatement (tests/golden/make_golden.py).
//
// Build: g++ -O2 -std=c++17 -fopenmp -mavx2 -mfma -ffp-contract=off
//        -fno-builtin -fPIC -shared (see oracle/Makefile).

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

constexpr size_t kBlock = 32;          // quantize.rs:23
constexpr size_t kQ8Bytes = 4 + 32;    // quantize.rs:25
constexpr size_t kQ4Bytes = 4 + 16;    // quantize.rs:27

enum Dtype : int { DT_Q8_0 = 1, DT_Q4_0 = 2 };  // storage tags, format.rs:37-39

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

// Status codes shared with the product's C ABI numbering.
enum : int { OK = 0, E_IO = 1, E_SHAPE = 2, E_FORMAT = 3, E_MODEL = 4 };

inline float read_f32_le(const uint8_t* p) {  // quantize.rs:63
  float f;
  std::memcpy(&f, p, 4);
  return f;
}

// f32::max — returns the non-NaN operand when one is NaN (IEEE maxNum).
inline float rmax(float a, float b) { return std::fmax(a, b); }

// Rust `f32::clamp` then saturating `as` cast to an integer: NaN -> 0.
inline int clamp_cast(float v, float lo, float hi) {
  if (std::isnan(v)) return 0;
  float c = v < lo ? lo : (v > hi ? hi : v);
  return static_cast<int>(c);
}

// ---------------------------------------------------------------------------
// quantize.rs:78-96 — Q8_0 block quantizer (bit-exact contract).
void quantize_q8_0_impl(const float* x, size_t n, uint8_t* out) {
  // Blocks are independent: parallel over blocks gives identical bytes.
#pragma omp parallel for schedule(static) if (n >= (1u << 20))
  for (size_t b = 0; b < n / kBlock; ++b) {
    const float* blk = x + b * kBlock;
    uint8_t* o = out + b * kQ8Bytes;
    float amax = 0.0f;
    for (size_t i = 0; i < kBlock; ++i) amax = rmax(amax, std::fabs(blk[i]));
    float d = amax / 127.0f;
    std::memcpy(o, &d, 4);
    if (d == 0.0f) {
      std::memset(o + 4, 0, kBlock);
    } else {
      float id = 1.0f / d;
      for (size_t i = 0; i < kBlock; ++i) {
        float r = std::round(blk[i] * id);  // Rust round: half away from zero
        int q = clamp_cast(r, -127.0f, 127.0f);
        o[4 + i] = static_cast<uint8_t>(static_cast<int8_t>(q));
      }
    }
  }
}

// quantize.rs:120-143 — Q4_0 block quantizer (bit-exact contract).
void quantize_q4_0_impl(const float* x, size_t n, uint8_t* out) {
  // Blocks are independent: parallel over blocks gives identical bytes.
#pragma omp parallel for schedule(static) if (n >= (1u << 20))
  for (size_t b = 0; b < n / kBlock; ++b) {
    const float* blk = x + b * kBlock;
    uint8_t* o = out + b * kQ4Bytes;
    float amax = 0.0f;
    for (size_t i = 0; i < kBlock; ++i) amax = rmax(amax, std::fabs(blk[i]));
    float d = amax / 8.0f;
    std::memcpy(o, &d, 4);
    uint8_t packed[16] = {0};
    if (d != 0.0f) {
      float id = 1.0f / d;
      for (size_t i = 0; i < kBlock; ++i) {
        int q = clamp_cast(std::round(blk[i] * id), -8.0f, 7.0f);
        uint8_t code = static_cast<uint8_t>(q + 8);
        if (i % 2 == 0)
          packed[i / 2] |= code;
        else
          packed[i / 2] |= static_cast<uint8_t>(code << 4);
      }
    }
    std::memcpy(o + 4, packed, 16);
  }
}

// quantize.rs:99-117
void dequantize_q8_0_impl(const uint8_t* bytes, size_t nblocks, float* out) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t* blk = bytes + b * kQ8Bytes;
    float d = read_f32_le(blk);
    for (size_t i = 0; i < kBlock; ++i)
      out[b * kBlock + i] = static_cast<float>(static_cast<int8_t>(blk[4 + i])) * d;
  }
}

// quantize.rs:146-166
void dequantize_q4_0_impl(const uint8_t* bytes, size_t nblocks, float* out) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t* blk = bytes + b * kQ4Bytes;
    float d = read_f32_le(blk);
    for (size_t i = 0; i < kBlock / 2; ++i) {
      uint8_t byte = blk[4 + i];
      out[b * kBlock + 2 * i] = static_cast<float>(static_cast<int>(byte & 0x0F) - 8) * d;
      out[b * kBlock + 2 * i + 1] = static_cast<float>(static_cast<int>(byte >> 4) - 8) * d;
    }
  }
}

// quantize.rs:252-264 — scalar Q8_0 row kernel.
float row_q8_0_scalar(const uint8_t* row, const float* x, size_t nblocks) {
  float acc = 0.0f;
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t* blk = row + b * kQ8Bytes;
    float d = read_f32_le(blk);
    float sum = 0.0f;
    for (size_t i = 0; i < kBlock; ++i)
      sum += static_cast<float>(static_cast<int8_t>(blk[4 + i])) * x[b * kBlock + i];
    acc += d * sum;
  }
  return acc;
}

// quantize.rs:266-280 — scalar Q4_0 row kernel.
float row_q4_0_scalar(const uint8_t* row, const float* x, size_t nblocks) {
  float acc = 0.0f;
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t* blk = row + b * kQ4Bytes;
    float d = read_f32_le(blk);
    const float* xb = x + b * kBlock;
    float sum = 0.0f;
    for (size_t i = 0; i < kBlock / 2; ++i) {
      uint8_t byte = blk[4 + i];
      sum += static_cast<float>(static_cast<int>(byte & 0x0F) - 8) * xb[2 * i] +
             static_cast<float>(static_cast<int>(byte >> 4) - 8) * xb[2 * i + 1];
    }
    acc += d * sum;
  }
  return acc;
}

// quantize.rs:295-304 — horizontal sum of 8 lanes, same shuffle tree.
__attribute__((target("avx2,fma"))) inline float hsum_ps(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 s = _mm_add_ps(lo, hi);
  __m128 shuf = _mm_movehdup_ps(s);
  __m128 sums = _mm_add_ps(s, shuf);
  __m128 shuf2 = _mm_movehl_ps(shuf, sums);
  return _mm_cvtss_f32(_mm_add_ss(sums, shuf2));
}

// quantize.rs:312-326 — four 8-lane groups, mul then three FMAs.
__attribute__((target("avx2,fma"))) inline float block_dot(__m256i q, const float* xp) {
  __m128i lo = _mm256_castsi256_si128(q);
  __m128i hi = _mm256_extracti128_si256(q, 1);
  __m256 q0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(lo));
  __m256 q1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(lo, 8)));
  __m256 q2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(hi));
  __m256 q3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(hi, 8)));
  __m256 s = _mm256_mul_ps(q0, _mm256_loadu_ps(xp));
  s = _mm256_fmadd_ps(q1, _mm256_loadu_ps(xp + 8), s);
  s = _mm256_fmadd_ps(q2, _mm256_loadu_ps(xp + 16), s);
  s = _mm256_fmadd_ps(q3, _mm256_loadu_ps(xp + 24), s);
  return hsum_ps(s);
}

// quantize.rs:336-349
__attribute__((target("avx2,fma"))) float row_q8_0_avx2(const uint8_t* row, const float* x,
                                                        size_t nblocks) {
  float acc = 0.0f;
  const uint8_t* rp = row;
  const float* xp = x;
  for (size_t b = 0; b < nblocks; ++b) {
    float d = read_f32_le(rp);
    __m256i q = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(rp + 4));
    acc += d * block_dot(q, xp);
    rp += kQ8Bytes;
    xp += 32;
  }
  return acc;
}

// quantize.rs:364-385 — nibble unpack with and / srli_epi16 / unpacklo-hi.
__attribute__((target("avx2,fma"))) float row_q4_0_avx2(const uint8_t* row, const float* x,
                                                        size_t nblocks) {
  float acc = 0.0f;
  const uint8_t* rp = row;
  const float* xp = x;
  const __m128i nibble_mask = _mm_set1_epi8(0x0F);
  const __m256i eight = _mm256_set1_epi8(8);
  for (size_t b = 0; b < nblocks; ++b) {
    float d = read_f32_le(rp);
    __m128i packed = _mm_loadu_si128(reinterpret_cast<const __m128i*>(rp + 4));
    __m128i lo = _mm_and_si128(packed, nibble_mask);
    __m128i hi = _mm_and_si128(_mm_srli_epi16(packed, 4), nibble_mask);
    __m128i e0 = _mm_unpacklo_epi8(lo, hi);
    __m128i e1 = _mm_unpackhi_epi8(lo, hi);
    __m256i q = _mm256_sub_epi8(_mm256_set_m128i(e1, e0), eight);
    acc += d * block_dot(q, xp);
    rp += kQ4Bytes;
    xp += 32;
  }
  return acc;
}

// tensor.rs:114-116 — sequential scalar dot.
float dot_scalar(const float* a, const float* b, size_t n) {
  float s = 0.0f;
  for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

// tensor.rs:125-154 — two 8-lane FMA accumulators, scalar tail.
__attribute__((target("avx2,fma"))) float dot_avx2(const float* a, const float* b, size_t n) {
  __m256 acc0 = _mm256_setzero_ps();
  __m256 acc1 = _mm256_setzero_ps();
  size_t i = 0;
  while (i + 16 <= n) {
    __m256 a0 = _mm256_loadu_ps(a + i);
    __m256 b0 = _mm256_loadu_ps(b + i);
    __m256 a1 = _mm256_loadu_ps(a + i + 8);
    __m256 b1 = _mm256_loadu_ps(b + i + 8);
    acc0 = _mm256_fmadd_ps(a0, b0, acc0);
    acc1 = _mm256_fmadd_ps(a1, b1, acc1);
    i += 16;
  }
  float total = hsum_ps(_mm256_add_ps(acc0, acc1));
  for (size_t j = i; j < n; ++j) total += a[j] * b[j];
  return total;
}

bool g_simd = true;  // tensor.rs:85-99 runtime dispatch; AVX2 on x86 hosts
int g_threads = 0;   // 0 = OpenMP default (all cores), like rayon's global pool

inline float dot(const float* a, const float* b, size_t n) {  // tensor.rs:102-111
  return g_simd ? dot_avx2(a, b, n) : dot_scalar(a, b, n);
}

inline int nthreads() { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

// quantize.rs:215-249 — rows in parallel, one row per task.
void qmatvec(int dtype, const uint8_t* data, size_t rows, size_t cols, const float* x, float* y) {
  size_t nb = cols / kBlock;
  size_t bb = dtype == DT_Q8_0 ? kQ8Bytes : kQ4Bytes;
  size_t row_bytes = nb * bb;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long r = 0; r < static_cast<long>(rows); ++r) {
    const uint8_t* row = data + r * row_bytes;
    float v;
    if (dtype == DT_Q8_0)
      v = g_simd ? row_q8_0_avx2(row, x, nb) : row_q8_0_scalar(row, x, nb);
    else
      v = g_simd ? row_q4_0_avx2(row, x, nb) : row_q4_0_scalar(row, x, nb);
    y[r] = v;
  }
}

// tensor.rs:181-192
void matvec_f32(const float* w, size_t rows, size_t cols, const float* x, float* y) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long r = 0; r < static_cast<long>(rows); ++r) y[r] = dot(w + r * cols, x, cols);
}

// tensor.rs:219-227
void rmsnorm(const float* x, const float* w, float eps, size_t n, float* out) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
  ss = ss / static_cast<float>(n);
  float inv = 1.0f / std::sqrt(ss + eps);
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv * w[i];
}

// tensor.rs:211-215
inline float silu1(float v) { return v / (1.0f + std::exp(-v)); }

// tensor.rs:230-245
void softmax(float* x, size_t n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = rmax(mx, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    x[i] = std::exp(x[i] - mx);
    sum += x[i];
  }
  if (sum > 0.0f)
    for (size_t i = 0; i < n; ++i) x[i] /= sum;
}

// model.rs:146 / model.rs:178 — identical f32 expression in both places.
inline void rope_angle(size_t pos, size_t i, size_t head_dim, float theta, float* s, float* c) {
  float freq = 1.0f / std::pow(theta, 2.0f * static_cast<float>(i) / static_cast<float>(head_dim));
  float angle = static_cast<float>(pos) * freq;
  *s = std::sin(angle);
  *c = std::cos(angle);
}

// model.rs:140-155 — on-the-fly RoPE (reference for the tables).
void apply_rope(float* x, size_t pos, size_t n_heads, size_t head_dim, float theta) {
  size_t half = head_dim / 2;
  for (size_t h = 0; h < n_heads; ++h) {
    float* head = x + h * head_dim;
    for (size_t i = 0; i < half; ++i) {
      float s, c;
      rope_angle(pos, i, head_dim, theta, &s, &c);
      float x1 = head[i], x2 = head[i + half];
      head[i] = x1 * c - x2 * s;
      head[i + half] = x2 * c + x1 * s;
    }
  }
}

struct Rope {  // model.rs:162-202
  std::vector<float> cos, sin;
  size_t half = 0;
  void build(size_t head_dim, size_t max_seq, float theta) {
    half = head_dim / 2;
    cos.assign(max_seq * half, 0.0f);
    sin.assign(max_seq * half, 0.0f);
    for (size_t pos = 0; pos < max_seq; ++pos)
      for (size_t i = 0; i < half; ++i)
        rope_angle(pos, i, head_dim, theta, &sin[pos * half + i], &cos[pos * half + i]);
  }
  void apply(float* x, size_t n, size_t pos) const {
    const float* c = &cos[pos * half];
    const float* s = &sin[pos * half];
    for (size_t h = 0; h < n / (2 * half); ++h) {
      float* head = x + h * 2 * half;
      for (size_t i = 0; i < half; ++i) {
        float x1 = head[i], x2 = head[i + half];
        head[i] = x1 * c[i] - x2 * s[i];
        head[i + half] = x2 * c[i] + x1 * s[i];
      }
    }
  }
};

// model.rs:206-216
void per_head_norm(float* x, size_t n, const float* w, float eps, size_t hd) {
  for (size_t h = 0; h < n / hd; ++h) {
    float* head = x + h * hd;
    float ss = 0.0f;
    for (size_t i = 0; i < hd; ++i) ss += head[i] * head[i];
    ss = ss / static_cast<float>(hd);
    float inv = 1.0f / std::sqrt(ss + eps);
    for (size_t i = 0; i < hd; ++i) head[i] = head[i] * inv * w[i];
  }
}

struct Config {  // model.rs:29-45
  size_t hidden = 0, inter = 0, n_layers = 0, n_heads = 0, n_kv = 0, head_dim = 0, vocab = 0,
         max_seq = 0;
  float theta = 10000.0f, eps = 1e-6f;
  bool qkv_bias = false;
  std::string dtype = "f32";
};

// Heads of attend() in parallel (off by default: the reference loops over
// them on one thread). Each head's arithmetic is the same either way, so the
// output is bit-identical; checks over long histories turn it on to finish
// sooner, the timed CPU baseline leaves it off.
bool g_attn_parallel = false;

// model.rs:223-248 — serial over heads; scores, softmax, weighted V sum.
void attend(const float* q, const float* k, const float* v, size_t len, const Config& c,
            float* out) {
  size_t hd = c.head_dim, kv_dim = c.n_kv * hd, group = c.n_heads / c.n_kv;
  float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  std::fill(out, out + c.n_heads * hd, 0.0f);
  auto head = [&](size_t h, float* scores) {
    const float* qh = q + h * hd;
    size_t off = (h / group) * hd;
    for (size_t t = 0; t < len; ++t) scores[t] = dot(qh, k + t * kv_dim + off, hd) * scale;
    softmax(scores, len);
    float* oh = out + h * hd;
    for (size_t t = 0; t < len; ++t) {
      const float* vt = v + t * kv_dim + off;
      float w = scores[t];
      for (size_t i = 0; i < hd; ++i) oh[i] += w * vt[i];
    }
  };
  if (!g_attn_parallel) {
    std::vector<float> scores(len);
    for (size_t h = 0; h < c.n_heads; ++h) head(h, scores.data());
    return;
  }
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> scores(len);
#pragma omp for schedule(dynamic, 1)
    for (long h = 0; h < static_cast<long>(c.n_heads); ++h) head((size_t)h, scores.data());
  }
}

struct Linear {  // model.rs:50-63
  bool quant = false;
  int dtype = 0;
  size_t rows = 0, cols = 0;
  std::vector<float> f;
  std::vector<uint8_t> q;
  void matvec(const float* x, float* y) const {
    if (quant)
      qmatvec(dtype, q.data(), rows, cols, x, y);
    else
      matvec_f32(f.data(), rows, cols, x, y);
  }
};

struct Layer {  // model.rs:67-84
  std::vector<float> attn_norm, ffn_norm, q_bias, k_bias, v_bias, q_norm, k_norm;
  Linear q, k, v, o, gate, up, down;
};

struct Tensor {  // format.rs:43-46 WeightTensor
  int tag = 0;   // 0 f32, 1 q8_0, 2 q4_0
  std::vector<uint64_t> shape;
  std::vector<uint8_t> bytes;
};

struct Model {
  Config cfg;
  std::vector<float> embed;  // [vocab, hidden]
  std::vector<Layer> layers;
  std::vector<float> final_norm;
  Linear lm_head;
  Rope rope;
  std::map<std::string, Tensor> pending;  // named tensors before assemble()
};

struct Cache {  // model.rs:100-131
  std::vector<std::vector<float>> k, v;
  size_t len = 0;
};

int take_vec(Model& m, const std::string& name, bool required, std::vector<float>* out,
             size_t expect_len) {
  auto it = m.pending.find(name);
  if (it == m.pending.end()) {
    if (required) return fail(E_MODEL, "missing tensor `" + name + "`");
    out->clear();
    return OK;
  }
  const Tensor& t = it->second;
  if (t.tag != 0 || t.shape.size() != 1)
    return fail(E_MODEL, "tensor `" + name + "` must be a 1-D f32 vector");
  out->resize(t.shape[0]);
  std::memcpy(out->data(), t.bytes.data(), t.bytes.size());
  if (expect_len && out->size() != expect_len)
    return fail(E_SHAPE, "tensor `" + name + "` has wrong length");
  return OK;
}

int take_linear(Model& m, const std::string& name, Linear* out) {
  auto it = m.pending.find(name);
  if (it == m.pending.end()) return fail(E_MODEL, "missing tensor `" + name + "`");
  const Tensor& t = it->second;
  if (t.shape.size() != 2) return fail(E_MODEL, "tensor `" + name + "` must be 2-D");
  out->rows = t.shape[0];
  out->cols = t.shape[1];
  if (t.tag == 0) {
    out->quant = false;
    out->f.resize(out->rows * out->cols);
    std::memcpy(out->f.data(), t.bytes.data(), t.bytes.size());
  } else {
    out->quant = true;
    out->dtype = t.tag;
    out->q = t.bytes;
  }
  return OK;
}

// model.rs:522-574
int assemble(Model& m) {
  const Config& c = m.cfg;
  if (c.head_dim % 2 != 0) return fail(E_MODEL, "head_dim must be even (RoPE)");
  if (c.n_kv == 0 || c.n_heads % c.n_kv != 0)
    return fail(E_MODEL, "n_heads must be a multiple of n_kv_heads");
  auto it = m.pending.find("model.embed_tokens.weight");
  if (it == m.pending.end()) return fail(E_MODEL, "missing tensor `model.embed_tokens.weight`");
  if (it->second.tag != 0 || it->second.shape.size() != 2)
    return fail(E_MODEL, "model.embed_tokens.weight must be 2-D f32");
  m.embed.resize(it->second.bytes.size() / 4);
  std::memcpy(m.embed.data(), it->second.bytes.data(), it->second.bytes.size());
  m.layers.assign(c.n_layers, Layer());
  int rc;
  for (size_t i = 0; i < c.n_layers; ++i) {
    std::string p = "model.layers." + std::to_string(i);
    Layer& L = m.layers[i];
    if ((rc = take_vec(m, p + ".input_layernorm.weight", true, &L.attn_norm, 0))) return rc;
    if ((rc = take_linear(m, p + ".self_attn.q_proj.weight", &L.q))) return rc;
    if ((rc = take_linear(m, p + ".self_attn.k_proj.weight", &L.k))) return rc;
    if ((rc = take_linear(m, p + ".self_attn.v_proj.weight", &L.v))) return rc;
    if ((rc = take_linear(m, p + ".self_attn.o_proj.weight", &L.o))) return rc;
    if ((rc = take_vec(m, p + ".self_attn.q_proj.bias", false, &L.q_bias, 0))) return rc;
    if ((rc = take_vec(m, p + ".self_attn.k_proj.bias", false, &L.k_bias, 0))) return rc;
    if ((rc = take_vec(m, p + ".self_attn.v_proj.bias", false, &L.v_bias, 0))) return rc;
    if ((rc = take_vec(m, p + ".self_attn.q_norm.weight", false, &L.q_norm, 0))) return rc;
    if ((rc = take_vec(m, p + ".self_attn.k_norm.weight", false, &L.k_norm, 0))) return rc;
    if ((rc = take_vec(m, p + ".post_attention_layernorm.weight", true, &L.ffn_norm, 0)))
      return rc;
    if ((rc = take_linear(m, p + ".mlp.gate_proj.weight", &L.gate))) return rc;
    if ((rc = take_linear(m, p + ".mlp.up_proj.weight", &L.up))) return rc;
    if ((rc = take_linear(m, p + ".mlp.down_proj.weight", &L.down))) return rc;
  }
  if ((rc = take_vec(m, "model.norm.weight", true, &m.final_norm, 0))) return rc;
  if (m.pending.count("lm_head.weight")) {
    if ((rc = take_linear(m, "lm_head.weight", &m.lm_head))) return rc;
  } else {  // tied embeddings: model.rs:562-565
    m.lm_head.quant = false;
    m.lm_head.rows = c.vocab;
    m.lm_head.cols = c.hidden;
    m.lm_head.f = m.embed;
  }
  m.rope.build(c.head_dim, c.max_seq, c.theta);
  m.pending.clear();
  return OK;
}

// model.rs:273-318 — one decoder step at `pos`, appending K/V.
int forward_token(const Model& m, uint32_t tok, size_t pos, Cache& cache, float* logits) {
  const Config& c = m.cfg;
  if (tok >= c.vocab) return fail(E_SHAPE, "row index out of bounds");
  size_t H = c.hidden, qd = c.n_heads * c.head_dim, kvd = c.n_kv * c.head_dim, I = c.inter;
  std::vector<float> x(m.embed.begin() + tok * H, m.embed.begin() + (tok + 1) * H);
  std::vector<float> xn(H), q(qd), k(kvd), v(kvd), att(qd), proj(H), g(I), u(I), hid(I), dn(H);
  for (size_t li = 0; li < c.n_layers; ++li) {
    const Layer& L = m.layers[li];
    rmsnorm(x.data(), L.attn_norm.data(), c.eps, H, xn.data());
    L.q.matvec(xn.data(), q.data());
    L.k.matvec(xn.data(), k.data());
    L.v.matvec(xn.data(), v.data());
    if (!L.q_bias.empty()) for (size_t i = 0; i < qd; ++i) q[i] += L.q_bias[i];
    if (!L.k_bias.empty()) for (size_t i = 0; i < kvd; ++i) k[i] += L.k_bias[i];
    if (!L.v_bias.empty()) for (size_t i = 0; i < kvd; ++i) v[i] += L.v_bias[i];
    if (!L.q_norm.empty()) per_head_norm(q.data(), qd, L.q_norm.data(), c.eps, c.head_dim);
    if (!L.k_norm.empty()) per_head_norm(k.data(), kvd, L.k_norm.data(), c.eps, c.head_dim);
    m.rope.apply(q.data(), qd, pos);
    m.rope.apply(k.data(), kvd, pos);
    cache.k[li].insert(cache.k[li].end(), k.begin(), k.end());
    cache.v[li].insert(cache.v[li].end(), v.begin(), v.end());
    attend(q.data(), cache.k[li].data(), cache.v[li].data(), pos + 1, c, att.data());
    L.o.matvec(att.data(), proj.data());
    for (size_t i = 0; i < H; ++i) x[i] += proj[i];
    rmsnorm(x.data(), L.ffn_norm.data(), c.eps, H, xn.data());
    L.gate.matvec(xn.data(), g.data());
    L.up.matvec(xn.data(), u.data());
    for (size_t i = 0; i < I; ++i) hid[i] = silu1(g[i]);
    for (size_t i = 0; i < I; ++i) hid[i] *= u[i];
    L.down.matvec(hid.data(), dn.data());
    for (size_t i = 0; i < H; ++i) x[i] += dn[i];
  }
  rmsnorm(x.data(), m.final_norm.data(), c.eps, H, xn.data());
  m.lm_head.matvec(xn.data(), logits);
  return OK;
}

// model.rs:337-424 — one-shot causal sweep (returns per-position states).
int forward_full_states(const Model& m, const uint32_t* toks, size_t n, float* states) {
  const Config& c = m.cfg;
  if (n == 0) return fail(E_MODEL, "empty token sequence");
  if (n > c.max_seq) return fail(E_MODEL, "sequence exceeds max_seq_len");
  size_t H = c.hidden, hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv * hd, I = c.inter;
  std::vector<std::vector<float>> xs(n);
  for (size_t t = 0; t < n; ++t) {
    if (toks[t] >= c.vocab) return fail(E_SHAPE, "row index out of bounds");
    xs[t].assign(m.embed.begin() + toks[t] * H, m.embed.begin() + (toks[t] + 1) * H);
  }
  std::vector<float> xn(H), att(qd), proj(H), g(I), u(I), hid(I), dn(H);
  for (const Layer& L : m.layers) {
    std::vector<std::vector<float>> qs(n, std::vector<float>(qd)), ks(n, std::vector<float>(kvd)),
        vs(n, std::vector<float>(kvd));
    for (size_t t = 0; t < n; ++t) {
      rmsnorm(xs[t].data(), L.attn_norm.data(), c.eps, H, xn.data());
      L.q.matvec(xn.data(), qs[t].data());
      L.k.matvec(xn.data(), ks[t].data());
      L.v.matvec(xn.data(), vs[t].data());
      if (!L.q_bias.empty()) for (size_t i = 0; i < qd; ++i) qs[t][i] += L.q_bias[i];
      if (!L.k_bias.empty()) for (size_t i = 0; i < kvd; ++i) ks[t][i] += L.k_bias[i];
      if (!L.v_bias.empty()) for (size_t i = 0; i < kvd; ++i) vs[t][i] += L.v_bias[i];
    }
    for (size_t t = 0; t < n; ++t) {
      if (!L.q_norm.empty()) per_head_norm(qs[t].data(), qd, L.q_norm.data(), c.eps, hd);
      m.rope.apply(qs[t].data(), qd, t);
    }
    for (size_t t = 0; t < n; ++t) {
      if (!L.k_norm.empty()) per_head_norm(ks[t].data(), kvd, L.k_norm.data(), c.eps, hd);
      m.rope.apply(ks[t].data(), kvd, t);
    }
    std::vector<float> kf(n * kvd), vf(n * kvd);
    for (size_t t = 0; t < n; ++t) {
      std::memcpy(&kf[t * kvd], ks[t].data(), kvd * 4);
      std::memcpy(&vf[t * kvd], vs[t].data(), kvd * 4);
    }
    for (size_t t = 0; t < n; ++t) {
      attend(qs[t].data(), kf.data(), vf.data(), t + 1, c, att.data());
      L.o.matvec(att.data(), proj.data());
      for (size_t i = 0; i < H; ++i) xs[t][i] += proj[i];
    }
    for (size_t t = 0; t < n; ++t) {
      rmsnorm(xs[t].data(), L.ffn_norm.data(), c.eps, H, xn.data());
      L.gate.matvec(xn.data(), g.data());
      L.up.matvec(xn.data(), u.data());
      for (size_t i = 0; i < I; ++i) hid[i] = silu1(g[i]);
      for (size_t i = 0; i < I; ++i) hid[i] *= u[i];
      L.down.matvec(hid.data(), dn.data());
      for (size_t i = 0; i < H; ++i) xs[t][i] += dn[i];
    }
  }
  for (size_t t = 0; t < n; ++t) std::memcpy(states + t * H, xs[t].data(), H * 4);
  return OK;
}

// sampler.rs:10-17 — total_cmp order, ties to the lowest index.
inline int32_t total_key(float f) {
  int32_t b;
  std::memcpy(&b, &f, 4);
  return b ^ static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
}

uint32_t argmax(const float* x, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  int32_t bk = total_key(x[0]);
  for (size_t i = 1; i < n; ++i) {
    int32_t k = total_key(x[i]);
    if (k > bk) {
      bk = k;
      best = i;
    }
  }
  return static_cast<uint32_t>(best);
}

// ---------------------------------------------------------------------------
// format.rs:128-277 — hardened `.minq` reader.

struct Reader {
  FILE* f = nullptr;
  uint64_t pos = 0, len = 0;
  std::string path;
  int take(uint64_t n, const char* what) {
    uint64_t end = pos + n;
    if (end < pos) return fail(E_FORMAT, path + ": " + what + " length overflows");
    if (end > len)
      return fail(E_FORMAT, path + ": " + what + " claims " + std::to_string(n) +
                                " bytes at offset " + std::to_string(pos) + ", file is " +
                                std::to_string(len) + " bytes");
    pos = end;
    return OK;
  }
  bool read(void* dst, size_t n) { return n == 0 || std::fread(dst, 1, n, f) == n; }
};

// Minimal parser for the flat serde_json object of ModelConfig (model.rs:29-45).
int parse_config(const std::string& s, Config* c) {
  std::map<std::string, std::string> kv;
  size_t i = 0;
  auto skip = [&] { while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i; };
  skip();
  if (i >= s.size() || s[i] != '{') return fail(E_FORMAT, "config json: expected object");
  ++i;
  while (true) {
    skip();
    if (i < s.size() && s[i] == '}') break;
    if (i >= s.size() || s[i] != '"') return fail(E_FORMAT, "config json: expected key");
    size_t e = s.find('"', i + 1);
    if (e == std::string::npos) return fail(E_FORMAT, "config json: bad key");
    std::string key = s.substr(i + 1, e - i - 1);
    i = e + 1;
    skip();
    if (i >= s.size() || s[i] != ':') return fail(E_FORMAT, "config json: expected ':'");
    ++i;
    skip();
    std::string val;
    if (i < s.size() && s[i] == '"') {
      size_t e2 = s.find('"', i + 1);
      if (e2 == std::string::npos) return fail(E_FORMAT, "config json: bad string");
      val = s.substr(i, e2 - i + 1);
      i = e2 + 1;
    } else {
      size_t st = i;
      while (i < s.size() && s[i] != ',' && s[i] != '}') ++i;
      val = s.substr(st, i - st);
      while (!val.empty() && std::isspace(static_cast<unsigned char>(val.back()))) val.pop_back();
    }
    kv[key] = val;
    skip();
    if (i < s.size() && s[i] == ',') { ++i; continue; }
    if (i < s.size() && s[i] == '}') break;
    return fail(E_FORMAT, "config json: expected ',' or '}'");
  }
  const char* need[] = {"hidden_size", "intermediate_size", "n_layers", "n_heads", "n_kv_heads",
                        "head_dim", "vocab_size", "max_seq_len", "rope_theta", "rms_norm_eps",
                        "has_qkv_bias", "dtype"};
  for (const char* k : need)
    if (!kv.count(k)) return fail(E_FORMAT, std::string("config json: missing field `") + k + "`");
  auto u = [&](const char* k) { return static_cast<size_t>(std::strtoull(kv[k].c_str(), nullptr, 10)); };
  c->hidden = u("hidden_size");
  c->inter = u("intermediate_size");
  c->n_layers = u("n_layers");
  c->n_heads = u("n_heads");
  c->n_kv = u("n_kv_heads");
  c->head_dim = u("head_dim");
  c->vocab = u("vocab_size");
  c->max_seq = u("max_seq_len");
  c->theta = static_cast<float>(std::strtod(kv["rope_theta"].c_str(), nullptr));
  c->eps = static_cast<float>(std::strtod(kv["rms_norm_eps"].c_str(), nullptr));
  c->qkv_bias = kv["has_qkv_bias"] == "true";
  std::string d = kv["dtype"];
  c->dtype = d.size() >= 2 ? d.substr(1, d.size() - 2) : d;
  return OK;
}

int read_minq(const char* path, Model* m) {
  Reader r;
  r.path = path;
  r.f = std::fopen(path, "rb");
  if (!r.f) return fail(E_IO, std::string("io error: cannot open ") + path);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(r.f, std::fclose);
  std::fseek(r.f, 0, SEEK_END);
  r.len = static_cast<uint64_t>(std::ftell(r.f));
  std::fseek(r.f, 0, SEEK_SET);
  int rc;
  if ((rc = r.take(8, "magic"))) return rc;
  char magic[8];
  if (!r.read(magic, 8)) return fail(E_IO, "io error: short read");
  if (std::memcmp(magic, "MINQ0001", 8) != 0 && std::memcmp(magic, "MINFER01", 8) != 0)
    return fail(E_FORMAT, r.path + ": not a .minq/.minfer file (bad magic)");
  if ((rc = r.take(4, "config length"))) return rc;
  uint32_t cfg_len;
  if (!r.read(&cfg_len, 4)) return fail(E_IO, "io error: short read");
  if ((rc = r.take(cfg_len, "config json"))) return rc;
  std::string cfg(cfg_len, '\0');
  if (!r.read(&cfg[0], cfg_len)) return fail(E_IO, "io error: short read");
  if ((rc = parse_config(cfg, &m->cfg))) return rc;
  while (true) {
    uint8_t first;
    if (std::fread(&first, 1, 1, r.f) != 1) break;  // clean EOF
    if ((rc = r.take(4, "tensor name length"))) return rc;
    uint8_t rest[3];
    if (!r.read(rest, 3)) return fail(E_IO, "io error: short read");
    uint64_t name_len = first | (rest[0] << 8) | (rest[1] << 16) | (uint64_t(rest[2]) << 24);
    if ((rc = r.take(name_len, "tensor name"))) return rc;
    std::string name(name_len, '\0');
    if (!r.read(&name[0], name_len)) return fail(E_IO, "io error: short read");
    if ((rc = r.take(2, "tensor tag/ndim"))) return rc;
    uint8_t tag, ndim;
    if (!r.read(&tag, 1) || !r.read(&ndim, 1)) return fail(E_IO, "io error: short read");
    if ((rc = r.take(8ull * ndim, "tensor shape"))) return rc;
    Tensor t;
    t.tag = tag;
    t.shape.resize(ndim);
    if (!r.read(t.shape.data(), 8ull * ndim)) return fail(E_IO, "io error: short read");
    uint64_t numel = 1;
    for (uint64_t d : t.shape) {
      if (d != 0 && numel > UINT64_MAX / d)
        return fail(E_FORMAT, "tensor `" + name + "`: shape overflows usize");
      numel *= d;
    }
    if ((rc = r.take(8, "tensor data length"))) return rc;
    uint64_t data_len;
    if (!r.read(&data_len, 8)) return fail(E_IO, "io error: short read");
    uint64_t expected;
    if (tag == 0) {
      if (numel > UINT64_MAX / 4) return fail(E_FORMAT, "tensor `" + name + "`: byte count overflows");
      expected = numel * 4;
    } else if (tag == 1 || tag == 2) {
      if (ndim != 2) return fail(E_FORMAT, "quantized tensor `" + name + "` must be 2-D");
      uint64_t rows = t.shape[0], cols = t.shape[1];
      if (cols % kBlock != 0)
        return fail(E_FORMAT, "quantized tensor `" + name + "`: cols not block-aligned");
      uint64_t bb = tag == 1 ? kQ8Bytes : kQ4Bytes, nb = cols / kBlock;
      if (nb != 0 && rows > UINT64_MAX / nb) return fail(E_FORMAT, "byte count overflows");
      uint64_t blocks = rows * nb;
      if (blocks > UINT64_MAX / bb) return fail(E_FORMAT, "byte count overflows");
      expected = blocks * bb;
    } else {
      return fail(E_FORMAT, "tensor `" + name + "`: unknown storage tag " + std::to_string(tag));
    }
    if (data_len != expected)
      return fail(E_FORMAT, "tensor `" + name + "`: data length " + std::to_string(data_len) +
                                " != shape-derived " + std::to_string(expected));
    if ((rc = r.take(data_len, "tensor data"))) return rc;
    t.bytes.resize(data_len);
    if (!r.read(t.bytes.data(), data_len)) return fail(E_IO, "io error: short read");
    m->pending[name] = std::move(t);
  }
  return OK;
}

}  // namespace

// ===========================================================================
// C API (ctypes). Every function returns 0 on success or an error code with
// orc_last_error() describing it.

extern "C" {

const char* orc_last_error() { return g_err.c_str(); }
void orc_set_simd(int on) { g_simd = on != 0; }
void orc_set_threads(int n) { g_threads = n; }
void orc_set_attn_parallel(int on) { g_attn_parallel = on != 0; }
int orc_max_threads() { return omp_get_max_threads(); }

int orc_quantize(int dtype, const float* x, size_t n, uint8_t* out) {
  if (n % kBlock != 0)  // quantize.rs:67-75
    return fail(E_SHAPE, "quantization requires a multiple of 32 elements, got " + std::to_string(n));
  if (dtype == DT_Q8_0) quantize_q8_0_impl(x, n, out);
  else if (dtype == DT_Q4_0) quantize_q4_0_impl(x, n, out);
  else return fail(E_FORMAT, "unknown dtype");
  return OK;
}

int orc_dequantize(int dtype, const uint8_t* bytes, size_t nbytes, float* out, size_t nout) {
  size_t bb = dtype == DT_Q8_0 ? kQ8Bytes : kQ4Bytes;
  if (nbytes % bb != 0 || nout != nbytes / bb * kBlock)
    return fail(E_SHAPE, "dequantize: byte/output length mismatch");
  if (dtype == DT_Q8_0) dequantize_q8_0_impl(bytes, nbytes / bb, out);
  else dequantize_q4_0_impl(bytes, nbytes / bb, out);
  return OK;
}

int orc_qmatvec(int dtype, const uint8_t* data, size_t rows, size_t cols, const float* x,
                size_t xlen, float* y) {
  if (xlen != cols) return fail(E_SHAPE, "quantized matvec: cols vs input len");
  if (cols % kBlock) return fail(E_SHAPE, "cols not block-aligned");
  qmatvec(dtype, data, rows, cols, x, y);
  return OK;
}

int orc_qrow(int dtype, int simd, const uint8_t* row, const float* x, size_t cols, float* out) {
  size_t nb = cols / kBlock;
  if (dtype == DT_Q8_0) *out = simd ? row_q8_0_avx2(row, x, nb) : row_q8_0_scalar(row, x, nb);
  else *out = simd ? row_q4_0_avx2(row, x, nb) : row_q4_0_scalar(row, x, nb);
  return OK;
}

int orc_matvec_f32(const float* w, size_t rows, size_t cols, const float* x, size_t xlen,
                   float* y) {
  if (xlen != cols) return fail(E_SHAPE, "matvec: weight shape vs input len");
  matvec_f32(w, rows, cols, x, y);
  return OK;
}

float orc_dot(const float* a, const float* b, size_t n, int simd) {
  return simd ? dot_avx2(a, b, n) : dot_scalar(a, b, n);
}

void orc_rmsnorm(const float* x, const float* w, float eps, size_t n, float* out) {
  rmsnorm(x, w, eps, n, out);
}
void orc_silu(const float* x, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = silu1(x[i]);
}
void orc_softmax(float* x, size_t n) { softmax(x, n); }
void orc_apply_rope(float* x, size_t pos, size_t n_heads, size_t hd, float theta) {
  apply_rope(x, pos, n_heads, hd, theta);
}
void orc_rope_tables(size_t hd, size_t max_seq, float theta, float* cos_out, float* sin_out) {
  Rope r;
  r.build(hd, max_seq, theta);
  std::memcpy(cos_out, r.cos.data(), r.cos.size() * 4);
  std::memcpy(sin_out, r.sin.data(), r.sin.size() * 4);
}
void orc_rope_apply_tables(const float* cos_t, const float* sin_t, size_t half, float* x, size_t n,
                           size_t pos) {
  Rope r;
  r.half = half;
  r.cos.assign(cos_t, cos_t + (pos + 1) * half);
  r.sin.assign(sin_t, sin_t + (pos + 1) * half);
  r.apply(x, n, pos);
}
void orc_per_head_norm(float* x, size_t n, const float* w, float eps, size_t hd) {
  per_head_norm(x, n, w, eps, hd);
}
uint32_t orc_argmax(const float* x, size_t n) { return argmax(x, n); }

// attend() on a flat [len, n_kv*hd] history.
int orc_attend(const float* q, const float* k, const float* v, size_t len, size_t n_heads,
               size_t n_kv, size_t hd, float* out) {
  if (n_kv == 0 || n_heads % n_kv) return fail(E_SHAPE, "n_heads % n_kv_heads");
  Config c;
  c.n_heads = n_heads;
  c.n_kv = n_kv;
  c.head_dim = hd;
  attend(q, k, v, len, c, out);
  return OK;
}

// ---- model ----
void* orc_model_new(size_t hidden, size_t inter, size_t n_layers, size_t n_heads, size_t n_kv,
                    size_t head_dim, size_t vocab, size_t max_seq, float theta, float eps,
                    int qkv_bias) {
  Model* m = new Model();
  m->cfg.hidden = hidden;
  m->cfg.inter = inter;
  m->cfg.n_layers = n_layers;
  m->cfg.n_heads = n_heads;
  m->cfg.n_kv = n_kv;
  m->cfg.head_dim = head_dim;
  m->cfg.vocab = vocab;
  m->cfg.max_seq = max_seq;
  m->cfg.theta = theta;
  m->cfg.eps = eps;
  m->cfg.qkv_bias = qkv_bias != 0;
  return m;
}

int orc_model_add(void* h, const char* name, int tag, size_t ndim, const uint64_t* shape,
                  const void* data, size_t nbytes) {
  Model* m = static_cast<Model*>(h);
  Tensor t;
  t.tag = tag;
  t.shape.assign(shape, shape + ndim);
  t.bytes.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + nbytes);
  m->pending[name] = std::move(t);
  return OK;
}

int orc_model_finish(void* h) { return assemble(*static_cast<Model*>(h)); }

void* orc_model_load_minq(const char* path) {  // model.rs:711-715
  Model* m = new Model();
  if (read_minq(path, m) != OK || assemble(*m) != OK) {
    delete m;
    return nullptr;
  }
  return m;
}

// Parse only (no assemble): reports tensor count for the format tests.
int orc_read_minq_count(const char* path, size_t* count) {
  Model m;
  int rc = read_minq(path, &m);
  if (rc) return rc;
  *count = m.pending.size();
  return OK;
}

void orc_model_free(void* h) { delete static_cast<Model*>(h); }

int orc_model_config(void* h, size_t* out) {  // hidden, inter, L, nh, nkv, hd, vocab, max_seq
  const Config& c = static_cast<Model*>(h)->cfg;
  size_t v[8] = {c.hidden, c.inter, c.n_layers, c.n_heads, c.n_kv, c.head_dim, c.vocab, c.max_seq};
  std::memcpy(out, v, sizeof(v));
  return OK;
}

void* orc_cache_new(void* h) {
  Model* m = static_cast<Model*>(h);
  Cache* c = new Cache();
  c->k.resize(m->cfg.n_layers);
  c->v.resize(m->cfg.n_layers);
  return c;
}
void orc_cache_free(void* c) { delete static_cast<Cache*>(c); }
size_t orc_cache_len(void* c) { return static_cast<Cache*>(c)->len; }
void orc_cache_reset(void* c) {  // model.rs:124-130
  Cache* cc = static_cast<Cache*>(c);
  for (auto& v : cc->k) v.clear();
  for (auto& v : cc->v) v.clear();
  cc->len = 0;
}

// Pre-fill the cache with `n` positions of given K/V ([n_layers, n, kv_dim]),
// as a caller can through the public `LayerCache` fields (model.rs:103-114).
int orc_cache_fill(void* hm, void* hc, size_t n, const float* k, const float* v) {
  Model* m = static_cast<Model*>(hm);
  Cache* c = static_cast<Cache*>(hc);
  size_t kvd = m->cfg.n_kv * m->cfg.head_dim;
  for (size_t l = 0; l < m->cfg.n_layers; ++l) {
    c->k[l].assign(k + l * n * kvd, k + (l + 1) * n * kvd);
    c->v[l].assign(v + l * n * kvd, v + (l + 1) * n * kvd);
  }
  c->len = n;
  return OK;
}

int orc_cache_read(void* hm, void* hc, size_t layer, float* k, float* v) {
  Model* m = static_cast<Model*>(hm);
  Cache* c = static_cast<Cache*>(hc);
  if (layer >= m->cfg.n_layers) return fail(E_SHAPE, "layer out of range");
  std::memcpy(k, c->k[layer].data(), c->k[layer].size() * 4);
  std::memcpy(v, c->v[layer].data(), c->v[layer].size() * 4);
  return OK;
}

// model.rs:254-270 — token-by-token prefill/decode; logits of the last token.
int orc_forward(void* hm, void* hc, const uint32_t* toks, size_t n, float* logits) {
  Model* m = static_cast<Model*>(hm);
  Cache* c = static_cast<Cache*>(hc);
  if (n == 0) return fail(E_MODEL, "empty token sequence");
  for (size_t i = 0; i < n; ++i) {
    if (c->len >= m->cfg.max_seq)
      return fail(E_MODEL, "sequence exceeds max_seq_len (" + std::to_string(m->cfg.max_seq) + ")");
    int rc = forward_token(*m, toks[i], c->len, *c, logits);
    if (rc) return rc;
    c->len += 1;
  }
  return OK;
}

// model.rs:337-424
int orc_forward_full_states(void* hm, const uint32_t* toks, size_t n, float* states) {
  return forward_full_states(*static_cast<Model*>(hm), toks, n, states);
}

// model.rs:325-330
int orc_forward_full(void* hm, const uint32_t* toks, size_t n, float* logits) {
  Model* m = static_cast<Model*>(hm);
  size_t H = m->cfg.hidden;
  std::vector<float> st(n * H), xn(H);
  int rc = forward_full_states(*m, toks, n, st.data());
  if (rc) return rc;
  rmsnorm(&st[(n - 1) * H], m->final_norm.data(), m->cfg.eps, H, xn.data());
  m->lm_head.matvec(xn.data(), logits);
  return OK;
}

// ppl.rs:30-35: log-sum-exp in f64 over f32 differences from the f32 max.
double orc_nll(const float* logits, size_t n, uint32_t target) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = rmax(mx, logits[i]);
  double s = 0.0;
  for (size_t i = 0; i < n; ++i) s += std::exp((double)(logits[i] - mx));
  return (double)mx + std::log(s) - (double)logits[target];
}

// ppl.rs:44-103: non-overlapping windows of `context` tokens, each one
// forward_full_states sweep; position t in 1 .. len - 2 of a window scores
// window[t + 1]; nll summed in f64 in position order. window_ppl (n_windows
// doubles, or null) receives the cumulative ppl after each window (NaN while
// nothing is scored), as the reference's on_window callback sees it.
int orc_eval_ppl(void* hm, const uint32_t* toks, size_t n, size_t context, uint64_t* scored,
                 double* mean_nll, double* ppl, double* window_ppl) {
  Model* m = static_cast<Model*>(hm);
  if (n < 3) return fail(E_MODEL, "need at least 3 tokens to score, got " + std::to_string(n));
  if (context < 3) return fail(E_MODEL, "context must be >= 3, got " + std::to_string(context));
  if (context > m->cfg.max_seq)
    return fail(E_MODEL, "context " + std::to_string(context) + " exceeds max_seq_len (" +
                             std::to_string(m->cfg.max_seq) + ")");
  const size_t H = m->cfg.hidden, V = m->lm_head.rows;
  std::vector<float> st, xn(H), logits(V);
  double nll_sum = 0.0;
  size_t count = 0, wi = 0;
  for (size_t w0 = 0; w0 < n; w0 += context, ++wi) {
    const size_t len = std::min(context, n - w0);
    st.assign(len * H, 0.0f);
    int rc = forward_full_states(*m, toks + w0, len, st.data());
    if (rc) return rc;
    for (size_t t = 1; t + 1 < len; ++t) {
      rmsnorm(&st[t * H], m->final_norm.data(), m->cfg.eps, H, xn.data());
      m->lm_head.matvec(xn.data(), logits.data());
      nll_sum += orc_nll(logits.data(), V, toks[w0 + t + 1]);
      count += 1;
    }
    if (window_ppl) window_ppl[wi] = count ? std::exp(nll_sum / (double)count) : NAN;
  }
  if (count == 0) return fail(E_MODEL, "no scorable positions (sequence too short for context)");
  *scored = count;
  *mean_nll = nll_sum / (double)count;
  *ppl = std::exp(*mean_nll);
  return OK;
}

// ---------------------------------------------------------------------------
// Sampler (sampler.rs:20-109) and its RNG. The reference's StdRng is rand
// 0.8.8's, i.e. rand_chacha 0.3.1's ChaCha12Rng, seeded by rand_core 0.6.4's
// SeedableRng::seed_from_u64; neither crate is in the reference tree, so
// their published algorithms are restated here:
// * seed_from_u64: a PCG32 (XSH-RR) generator with state s advanced as
//   s = s * 6364136223846793005 + 11634580027462260723 before each output;
//   eight outputs, little-endian, form the 32-byte seed;
// * ChaCha12Rng::from_seed: key = the seed as eight little-endian words,
//   64-bit block counter 0 (state words 12, 13), stream 0 (words 14, 15);
//   each refill produces four consecutive 16-word blocks (64 words) and
//   next_u32 returns them in order;
// * gen::<f32>() (rand's Standard for f32): (next_u32() >> 8) * 2^-24.
// The ChaCha block function is pinned by the ChaCha20 keystream test vectors
// (all-zero key and nonce) in tests/test_oracle_sampler.py; the PCG
// expansion, the word layout and the float conversion are not pinned by any
// output of the reference.

struct StdRng {
  uint32_t key[8];
  uint64_t block = 0;
  uint32_t buf[64];
  unsigned idx = 64;
};

inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void chacha_block(const uint32_t key[8], uint64_t ctr, uint64_t stream, int rounds,
                  uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
  for (int i = 0; i < 8; ++i) s[4 + i] = key[i];
  s[12] = (uint32_t)ctr;
  s[13] = (uint32_t)(ctr >> 32);
  s[14] = (uint32_t)stream;
  s[15] = (uint32_t)(stream >> 32);
  uint32_t x[16];
  std::memcpy(x, s, sizeof(x));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < rounds; r += 2) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

void std_rng_seed(StdRng& g, uint64_t seed) {
  uint64_t st = seed;
  for (int i = 0; i < 8; ++i) {
    st = st * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xs = (uint32_t)(((st >> 18) ^ st) >> 27);
    const unsigned rot = (unsigned)(st >> 59);
    g.key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  g.block = 0;
  g.idx = 64;
}

uint32_t std_rng_u32(StdRng& g) {
  if (g.idx >= 64) {
    for (int b = 0; b < 4; ++b) chacha_block(g.key, g.block + b, 0, 12, g.buf + 16 * b);
    g.block += 4;
    g.idx = 0;
  }
  return g.buf[g.idx++];
}

float std_rng_f32(StdRng& g) { return (float)(std_rng_u32(g) >> 8) * (1.0f / 16777216.0f); }

struct Sampler {
  float temperature;
  size_t top_k;
  float top_p;
  StdRng rng;
};

// sampler.rs:47-109. The reference ranks the top-k survivors with
// select_nth_unstable_by and a stable sort on probability, which leaves the
// order of exactly equal probabilities at the top-k boundary unspecified;
// here (and on the GPU) equal probabilities rank by lower index.
uint32_t sampler_sample(Sampler& s, const float* logits, size_t n) {
  if (n == 0) return 0;
  if (s.temperature <= 0.0f || s.top_k == 1) return argmax(logits, n);
  std::vector<float> probs(n);
  for (size_t i = 0; i < n; ++i) probs[i] = logits[i] / s.temperature;
  softmax(probs.data(), n);
  if ((s.top_k == 0 || s.top_k >= n) && s.top_p >= 1.0f) {
    float r = std_rng_f32(s.rng);
    for (size_t i = 0; i < n; ++i) {
      r -= probs[i];
      if (r <= 0.0f) return (uint32_t)i;
    }
    return (uint32_t)(n - 1);
  }
  const size_t k = s.top_k == 0 ? n : std::min(s.top_k, n);
  std::vector<uint32_t> ranked(n);
  for (size_t i = 0; i < n; ++i) ranked[i] = (uint32_t)i;
  auto before = [&](uint32_t a, uint32_t b) {
    return probs[a] > probs[b] || (probs[a] == probs[b] && a < b);
  };
  if (k < n) {
    std::nth_element(ranked.begin(), ranked.begin() + (k - 1), ranked.end(), before);
    ranked.resize(k);
  }
  std::sort(ranked.begin(), ranked.end(), before);
  size_t cutoff = k;
  float cumulative = 0.0f;
  for (size_t r = 0; r < ranked.size(); ++r) {
    cumulative += probs[ranked[r]];
    if (cumulative >= s.top_p) {
      cutoff = r + 1;
      break;
    }
  }
  float total = 0.0f;
  for (size_t r = 0; r < cutoff; ++r) total += probs[ranked[r]];
  float rr = std_rng_f32(s.rng) * total;
  for (size_t r = 0; r < cutoff; ++r) {
    rr -= probs[ranked[r]];
    if (rr <= 0.0f) return ranked[r];
  }
  return ranked[cutoff - 1];
}

void* orc_sampler_new(float temperature, size_t top_k, float top_p, uint64_t seed) {
  Sampler* s = new Sampler{temperature, top_k, top_p, {}};
  std_rng_seed(s->rng, seed);
  return s;
}
void orc_sampler_free(void* s) { delete static_cast<Sampler*>(s); }
uint32_t orc_sampler_sample(void* s, const float* logits, size_t n) {
  return sampler_sample(*static_cast<Sampler*>(s), logits, n);
}
void orc_sampler_rng_u32(void* s, size_t n, uint32_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = std_rng_u32(static_cast<Sampler*>(s)->rng);
}
void orc_chacha_block(const uint32_t* key, uint64_t ctr, uint64_t stream, int rounds,
                      uint32_t* out) {
  chacha_block(key, ctr, stream, rounds, out);
}

}  // extern "C"
