"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, `__graft_entry__.smoke()` and
the CPU legs of bench.py as the parity reference / CPU baseline. The product package
`minq_b200` never imports this module.

Function names follow the reference (kn1g78/minq, Rust) so the tests read
like its own: `quantize_q8_0` (quantize.rs:78), `QuantizedTensor.matvec`
(quantize.rs:215), `Model.forward` (model.rs:254), `argmax` (sampler.rs:10).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

Q8_0 = 1
Q4_0 = 2
BLOCK_SIZE = 32
BLOCK_BYTES = {Q8_0: 36, Q4_0: 20}
DTYPE_NAMES = {"q8_0": Q8_0, "q4_0": Q4_0}


class OracleError(RuntimeError):
    """Error reported by the oracle (mirrors MinqError's variants by code)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.cpp"))
        ):
            build()
        L = C.CDLL(_LIB_PATH)
        P, S, I, F = C.c_void_p, C.c_size_t, C.c_int, C.c_float
        sig = {
            "orc_last_error": (C.c_char_p, []),
            "orc_set_simd": (None, [I]),
            "orc_set_threads": (None, [I]),
            "orc_set_attn_parallel": (None, [I]),
            "orc_max_threads": (I, []),
            "orc_quantize": (I, [I, P, S, P]),
            "orc_dequantize": (I, [I, P, S, P, S]),
            "orc_qmatvec": (I, [I, P, S, S, P, S, P]),
            "orc_qrow": (I, [I, I, P, P, S, P]),
            "orc_matvec_f32": (I, [P, S, S, P, S, P]),
            "orc_dot": (F, [P, P, S, I]),
            "orc_rmsnorm": (None, [P, P, F, S, P]),
            "orc_silu": (None, [P, S, P]),
            "orc_softmax": (None, [P, S]),
            "orc_apply_rope": (None, [P, S, S, S, F]),
            "orc_rope_tables": (None, [S, S, F, P, P]),
            "orc_rope_apply_tables": (None, [P, P, S, P, S, S]),
            "orc_per_head_norm": (None, [P, S, P, F, S]),
            "orc_argmax": (C.c_uint32, [P, S]),
            "orc_attend": (I, [P, P, P, S, S, S, S, P]),
            "orc_model_new": (P, [S, S, S, S, S, S, S, S, F, F, I]),
            "orc_model_add": (I, [P, C.c_char_p, I, S, P, P, S]),
            "orc_model_finish": (I, [P]),
            "orc_model_load_minq": (P, [C.c_char_p]),
            "orc_read_minq_count": (I, [C.c_char_p, P]),
            "orc_model_free": (None, [P]),
            "orc_model_config": (I, [P, P]),
            "orc_cache_new": (P, [P]),
            "orc_cache_free": (None, [P]),
            "orc_cache_len": (S, [P]),
            "orc_cache_reset": (None, [P]),
            "orc_cache_fill": (I, [P, P, S, P, P]),
            "orc_cache_read": (I, [P, P, S, P, P]),
            "orc_forward": (I, [P, P, P, S, P]),
            "orc_forward_full_states": (I, [P, P, S, P]),
            "orc_forward_full": (I, [P, P, S, P]),
            "orc_nll": (C.c_double, [P, S, C.c_uint32]),
            "orc_eval_ppl": (I, [P, P, S, S, P, P, P, P]),
            "orc_sampler_new": (P, [F, S, F, C.c_uint64]),
            "orc_sampler_free": (None, [P]),
            "orc_sampler_sample": (C.c_uint32, [P, P, S]),
            "orc_sampler_rng_u32": (None, [P, S, P]),
            "orc_chacha_block": (None, [P, C.c_uint64, C.c_uint64, I, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _check(rc: int):
    if rc != 0:
        raise OracleError(rc, lib().orc_last_error().decode())


def nll(logits, target: int) -> float:
    """ppl.rs:30-35: log-sum-exp (f64) minus the target's logit."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return float(lib().orc_nll(_p(x), x.size, target))


def set_simd(on: bool) -> None:
    """Select the AVX2+FMA kernels (the reference's x86 default) or scalar."""
    lib().orc_set_simd(1 if on else 0)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def set_attn_parallel(on: bool) -> None:
    """Run attend()'s heads on the OpenMP threads (bit-identical output; the
    reference, model.rs:223-248, and so the timed baseline, loop over them on
    one thread)."""
    lib().orc_set_attn_parallel(1 if on else 0)


def max_threads() -> int:
    return lib().orc_max_threads()


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def quantize(dtype: int, x) -> np.ndarray:
    x = _f32(x).ravel()
    out = np.zeros(x.size // BLOCK_SIZE * BLOCK_BYTES[dtype], dtype=np.uint8)
    _check(lib().orc_quantize(dtype, _p(x), x.size, _p(out)))
    return out


def quantize_q8_0(x) -> np.ndarray:  # quantize.rs:78
    return quantize(Q8_0, x)


def quantize_q4_0(x) -> np.ndarray:  # quantize.rs:120
    return quantize(Q4_0, x)


def dequantize(dtype: int, data: np.ndarray) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.zeros(data.size // BLOCK_BYTES[dtype] * BLOCK_SIZE, dtype=np.float32)
    _check(lib().orc_dequantize(dtype, _p(data), data.size, _p(out), out.size))
    return out


def qmatvec(dtype: int, data: np.ndarray, rows: int, cols: int, x) -> np.ndarray:
    """QuantizedTensor::matvec (quantize.rs:215)."""
    x = _f32(x)
    data = np.ascontiguousarray(data, dtype=np.uint8)
    y = np.zeros(rows, dtype=np.float32)
    _check(lib().orc_qmatvec(dtype, _p(data), rows, cols, _p(x), x.size, _p(y)))
    return y


def qrow(dtype: int, row: np.ndarray, x, simd: bool) -> float:
    x = _f32(x)
    row = np.ascontiguousarray(row, dtype=np.uint8)
    out = np.zeros(1, dtype=np.float32)
    _check(lib().orc_qrow(dtype, 1 if simd else 0, _p(row), _p(x), x.size, _p(out)))
    return float(out[0])


def matvec_f32(w: np.ndarray, x) -> np.ndarray:
    """tensor::matvec (tensor.rs:181)."""
    w = _f32(w)
    x = _f32(x)
    y = np.zeros(w.shape[0], dtype=np.float32)
    _check(lib().orc_matvec_f32(_p(w), w.shape[0], w.shape[1], _p(x), x.size, _p(y)))
    return y


def dot(a, b, simd: bool = True) -> float:
    a, b = _f32(a), _f32(b)
    return float(np.float32(lib().orc_dot(_p(a), _p(b), a.size, 1 if simd else 0)))


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    out = np.zeros_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), float(eps), x.size, _p(out))
    return out


def silu(x) -> np.ndarray:
    x = _f32(x)
    out = np.zeros_like(x)
    lib().orc_silu(_p(x), x.size, _p(out))
    return out


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_softmax(_p(x), x.size)
    return x


def apply_rope(x, pos: int, n_heads: int, head_dim: int, theta: float) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_apply_rope(_p(x), pos, n_heads, head_dim, float(theta))
    return x


def rope_tables(head_dim: int, max_seq: int, theta: float):
    half = head_dim // 2
    c = np.zeros(max_seq * half, dtype=np.float32)
    s = np.zeros(max_seq * half, dtype=np.float32)
    lib().orc_rope_tables(head_dim, max_seq, float(theta), _p(c), _p(s))
    return c.reshape(max_seq, half), s.reshape(max_seq, half)


def rope_apply_tables(cos, sin, x, pos: int) -> np.ndarray:
    cos, sin = _f32(cos), _f32(sin)
    x = _f32(x).copy()
    lib().orc_rope_apply_tables(_p(cos), _p(sin), cos.shape[1], _p(x), x.size, pos)
    return x


def per_head_norm(x, w, eps: float, head_dim: int) -> np.ndarray:
    x, w = _f32(x).copy(), _f32(w)
    lib().orc_per_head_norm(_p(x), x.size, _p(w), float(eps), head_dim)
    return x


def argmax(logits) -> int:  # sampler.rs:10
    x = _f32(logits)
    return int(lib().orc_argmax(_p(x), x.size))


def attend(q, k, v, length: int, n_heads: int, n_kv: int, head_dim: int) -> np.ndarray:
    """model.rs:223 — q [nh*hd], k/v [len, nkv*hd] flat."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.zeros(n_heads * head_dim, dtype=np.float32)
    _check(lib().orc_attend(_p(q), _p(k), _p(v), length, n_heads, n_kv, head_dim, _p(out)))
    return out


class Model:
    """Oracle model (model.rs:88-98), built from named tensors or a .minq file."""

    def __init__(self, handle, cfg: dict):
        self._h = handle
        self.config = cfg

    @classmethod
    def from_tensors(cls, cfg: dict, tensors: dict):
        """`tensors`: name -> (tag, shape, np.ndarray bytes-or-f32) like WeightTensor."""
        L = lib()
        h = L.orc_model_new(cfg["hidden_size"], cfg["intermediate_size"], cfg["n_layers"],
                            cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                            cfg["vocab_size"], cfg["max_seq_len"], float(cfg["rope_theta"]),
                            float(cfg["rms_norm_eps"]), 1 if cfg.get("has_qkv_bias") else 0)
        for name, (tag, shape, data) in tensors.items():
            data = np.ascontiguousarray(data)
            shp = np.asarray(shape, dtype=np.uint64)
            _check(L.orc_model_add(h, name.encode(), int(tag), len(shape), _p(shp), _p(data),
                                   data.nbytes))
        rc = L.orc_model_finish(h)
        if rc != 0:
            msg = L.orc_last_error().decode()
            L.orc_model_free(h)
            raise OracleError(rc, msg)
        return cls(h, dict(cfg))

    @classmethod
    def load_minq(cls, path: str):
        L = lib()
        h = L.orc_model_load_minq(str(path).encode())
        if not h:
            raise OracleError(-1, L.orc_last_error().decode())
        cfgv = np.zeros(8, dtype=np.uint64)
        L.orc_model_config(h, _p(cfgv))
        keys = ["hidden_size", "intermediate_size", "n_layers", "n_heads", "n_kv_heads",
                "head_dim", "vocab_size", "max_seq_len"]
        return cls(h, {k: int(v) for k, v in zip(keys, cfgv)})

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None

    def new_cache(self) -> "KVCache":
        return KVCache(self)

    def forward(self, tokens, cache: "KVCache") -> np.ndarray:
        """model.rs:254 — returns the last token's logits."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.config["vocab_size"], dtype=np.float32)
        _check(lib().orc_forward(self._h, cache._h, _p(t), t.size, _p(out)))
        return out

    def forward_full(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.config["vocab_size"], dtype=np.float32)
        _check(lib().orc_forward_full(self._h, _p(t), t.size, _p(out)))
        return out

    def forward_full_states(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((t.size, self.config["hidden_size"]), dtype=np.float32)
        _check(lib().orc_forward_full_states(self._h, _p(t), t.size, _p(out)))
        return out

    def eval_ppl(self, tokens, context: int) -> dict:
        """ppl.rs:44-103: windows of `context` tokens, one full-states sweep
        each; returns total_tokens, scored_positions, mean_nll, ppl and the
        cumulative ppl after each window (what on_window receives)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nw = max(1, -(-t.size // max(1, context)))
        win = np.full(nw, np.nan, dtype=np.float64)
        scored = np.zeros(1, dtype=np.uint64)
        mean, ppl = np.zeros(1, dtype=np.float64), np.zeros(1, dtype=np.float64)
        _check(lib().orc_eval_ppl(self._h, _p(t), t.size, context, _p(scored), _p(mean), _p(ppl),
                                  _p(win)))
        return {"total_tokens": int(t.size), "scored_positions": int(scored[0]),
                "mean_nll": float(mean[0]), "ppl": float(ppl[0]), "windows": win}


class Sampler:
    """sampler.rs:20-109 with rand 0.8's StdRng (ChaCha12, seed_from_u64)."""

    def __init__(self, temperature: float, top_k: int, top_p: float, seed: int):
        self._h = lib().orc_sampler_new(float(temperature), int(top_k), float(top_p), int(seed))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_sampler_free(self._h)
            self._h = None

    def sample(self, logits) -> int:
        x = np.ascontiguousarray(logits, dtype=np.float32)
        return int(lib().orc_sampler_sample(self._h, _p(x), x.size))

    def rng_u32(self, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.uint32)
        lib().orc_sampler_rng_u32(self._h, n, _p(out))
        return out


def chacha_block(key, counter: int, stream: int, rounds: int) -> np.ndarray:
    """One ChaCha block (16 words) for a key of 8 words."""
    k = np.ascontiguousarray(key, dtype=np.uint32)
    out = np.zeros(16, dtype=np.uint32)
    lib().orc_chacha_block(_p(k), counter, stream, rounds, _p(out))
    return out


class KVCache:
    """model.rs:110-131; K stored post-RoPE, position-major [len, nkv*hd]."""

    def __init__(self, model: Model):
        self.model = model
        self._h = lib().orc_cache_new(model._h)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_cache_free(self._h)
            self._h = None

    @property
    def len(self) -> int:
        return int(lib().orc_cache_len(self._h))

    def reset(self) -> None:
        lib().orc_cache_reset(self._h)

    def fill(self, k: np.ndarray, v: np.ndarray) -> None:
        """Pre-fill with [n_layers, n, kv_dim] K (post-RoPE) and V."""
        k, v = _f32(k), _f32(v)
        _check(lib().orc_cache_fill(self.model._h, self._h, k.shape[1], _p(k), _p(v)))

    def read(self, layer: int):
        cfg = self.model.config
        kvd = cfg["n_kv_heads"] * cfg["head_dim"]
        k = np.zeros((self.len, kvd), dtype=np.float32)
        v = np.zeros((self.len, kvd), dtype=np.float32)
        _check(lib().orc_cache_read(self.model._h, self._h, layer, _p(k), _p(v)))
        return k, v


def greedy_generate(model: Model, prompt, max_tokens: int):
    """engine.rs:52-88 with Sampler::greedy (sampler.rs:42,51-53).

    Returns (tokens, margins) where margins[i] is the top-1 minus top-2 logit
    gap at step i (used to diagnose a greedy flip)."""
    cache = model.new_cache()
    logits = model.forward(prompt, cache)
    out, margins = [], []
    for _ in range(max_tokens):
        tok = argmax(logits)
        part = np.partition(logits, -2)[-2:]
        margins.append(float(part[1] - part[0]))
        out.append(tok)
        logits = model.forward([tok], cache)
    return out, margins
