"""Python host API over the C ABI, mirroring the reference's Rust API so that
callers (and the parity tests) read like minq's own code:

  quantize_q8_0 / quantize_q4_0 / dequantize_*  quantize.rs:78-166
  QuantizedTensor(.from_tensor, .dequantize, .matvec)  quantize.rs:169-249
  Model(.load_minq, .from_tensors, .forward)     model.rs:88-318, 711
  KVCache(.new, .reset, .len)                    model.rs:110-131
  Sampler.greedy / Engine(.generate) / GenStats  sampler.rs:42, engine.rs:11-88
  argmax                                         sampler.rs:10

Every compute call runs on the GPU through libminq_cuda.so; there is no CPU
path. Device buffers for the op-level helpers come from torch (plumbing
only: the kernels never see torch types).
"""
from __future__ import annotations

import ctypes as C
import sys
from typing import Callable, Iterable

import numpy as np

from . import _lib
from ._lib import MinqError, check, lib
from .minq_format import ModelConfig, TAG_F32, TAG_Q4_0, TAG_Q8_0, BLOCK_SIZE, BLOCK_BYTES

__all__ = [
    "MinqError", "ModelConfig", "QuantDtype", "QuantizedTensor", "quantize_q8_0",
    "quantize_q4_0", "dequantize_q8_0", "dequantize_q4_0", "argmax", "Model", "KVCache",
    "Sampler", "Engine", "GenStats", "PplResult", "eval_ppl", "BLOCK_SIZE",
]

GenStats = _lib.GenStats
PplResult = _lib.PplResult


def _torch():
    import torch  # imported lazily; only used for device memory and streams
    return torch


def _dev_tensor(x, dtype):
    """Host array / torch tensor -> contiguous CUDA tensor of `dtype`."""
    torch = _torch()
    if isinstance(x, torch.Tensor):
        t = x
    else:
        t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(device="cuda", dtype=dtype).contiguous()


def _ptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _stream_ptr() -> C.c_void_p:
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class QuantDtype:
    """quantize.rs:29-61."""

    Q8_0 = TAG_Q8_0
    Q4_0 = TAG_Q4_0

    @staticmethod
    def block_bytes(dt: int) -> int:
        return BLOCK_BYTES[dt]

    @staticmethod
    def name(dt: int) -> str:
        return {TAG_Q8_0: "q8_0", TAG_Q4_0: "q4_0"}[dt]

    @staticmethod
    def parse(s: str) -> int:
        if s == "q8_0":
            return TAG_Q8_0
        if s == "q4_0":
            return TAG_Q4_0
        raise MinqError(_lib.ERR_FORMAT, f"unknown dtype `{s}` (expected q8_0 or q4_0)")


def quantize_device(dtype: int, x):
    """GPU quantizer: CUDA f32 tensor -> CUDA uint8 tensor of blocks."""
    torch = _torch()
    xt = _dev_tensor(x, torch.float32).reshape(-1)
    n = xt.numel()
    out = torch.empty(n // BLOCK_SIZE * BLOCK_BYTES[dtype], dtype=torch.uint8, device="cuda")
    check(lib().minq_quantize(dtype, _ptr(xt), n, _ptr(out), _stream_ptr()))
    return out


def _quantize_host(dtype: int, x) -> np.ndarray:
    return quantize_device(dtype, x).cpu().numpy()


def quantize_q8_0(x) -> np.ndarray:
    """quantize.rs:78 — returns the Q8_0 bytes (bit-identical), computed on the GPU."""
    return _quantize_host(TAG_Q8_0, x)


def quantize_q4_0(x) -> np.ndarray:
    """quantize.rs:120."""
    return _quantize_host(TAG_Q4_0, x)


def _dequantize(dtype: int, data) -> np.ndarray:
    torch = _torch()
    d = _dev_tensor(data, torch.uint8).reshape(-1)
    n_out = d.numel() // BLOCK_BYTES[dtype] * BLOCK_SIZE
    out = torch.empty(max(n_out, 1), dtype=torch.float32, device="cuda")
    check(lib().minq_dequantize(dtype, _ptr(d), d.numel(), _ptr(out), n_out, _stream_ptr()))
    return out[:n_out].cpu().numpy()


def dequantize_q8_0(data) -> np.ndarray:  # quantize.rs:99
    return _dequantize(TAG_Q8_0, data)


def dequantize_q4_0(data) -> np.ndarray:  # quantize.rs:146
    return _dequantize(TAG_Q4_0, data)


def argmax(logits) -> int:
    """sampler.rs:10 on the GPU (total_cmp order, lowest index on ties)."""
    torch = _torch()
    x = _dev_tensor(logits, torch.float32).reshape(-1)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib().minq_argmax(_ptr(x), x.numel(), _ptr(out), _stream_ptr()))
    return int(out.item()) & 0xFFFFFFFF


class QuantizedTensor:
    """quantize.rs:169-249: a [rows, cols] matrix in row-major block layout,
    held on the GPU for matvec."""

    def __init__(self, dtype: int, rows: int, cols: int, data):
        self.dtype, self.rows, self.cols = dtype, rows, cols
        torch = _torch()
        self._dev = _dev_tensor(data, torch.uint8).reshape(-1)
        if self._dev.numel() != rows * (cols // BLOCK_SIZE) * BLOCK_BYTES[dtype]:
            raise MinqError(_lib.ERR_SHAPE, "quantized tensor: data length does not match shape")

    @property
    def data(self) -> np.ndarray:
        return self._dev.cpu().numpy()

    @classmethod
    def from_tensor(cls, w, dtype: int) -> "QuantizedTensor":
        """quantize.rs:181-198."""
        w = np.asarray(w) if not hasattr(w, "shape") else w
        if len(w.shape) != 2 or w.shape[1] % BLOCK_SIZE != 0:
            raise MinqError(_lib.ERR_SHAPE, f"cannot quantize shape {list(w.shape)}: need 2-D "
                                            f"with cols % {BLOCK_SIZE} == 0")
        return cls(dtype, int(w.shape[0]), int(w.shape[1]), quantize_device(dtype, w))

    def dequantize(self) -> np.ndarray:
        return _dequantize(self.dtype, self._dev).reshape(self.rows, self.cols)

    def matvec_device(self, x_dev, y_dev=None):
        torch = _torch()
        if y_dev is None:
            y_dev = torch.empty(self.rows, dtype=torch.float32, device="cuda")
        check(lib().minq_qmatvec(self.dtype, _ptr(self._dev), self.rows, self.cols, _ptr(x_dev),
                                 x_dev.numel(), _ptr(y_dev), _stream_ptr()))
        return y_dev

    def matvec(self, x) -> np.ndarray:
        """quantize.rs:215 — y = W @ x on the GPU."""
        torch = _torch()
        return self.matvec_device(_dev_tensor(x, torch.float32).reshape(-1)).cpu().numpy()

    def matmul_device(self, x_dev, y_dev=None, ws_dev=None):
        """matvec of each row of x_dev [batch, cols] (batch 1..64) in one
        call: y_dev [batch, rows]."""
        torch = _torch()
        batch = int(x_dev.shape[0])
        if y_dev is None:
            y_dev = torch.empty(batch, self.rows, dtype=torch.float32, device="cuda")
        nbytes = lib().minq_qmatmul_workspace_bytes(batch, self.rows, self.cols)
        if ws_dev is None or ws_dev.numel() < nbytes:
            ws_dev = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        check(lib().minq_qmatmul(self.dtype, _ptr(self._dev), self.rows, self.cols, _ptr(x_dev),
                                 batch, _ptr(y_dev), _ptr(ws_dev), ws_dev.numel(), _stream_ptr()))
        return y_dev

    def matmul(self, x) -> np.ndarray:
        """quantize.rs:215 applied to every row of x [batch, cols]."""
        torch = _torch()
        xd = _dev_tensor(x, torch.float32)
        if xd.dim() != 2 or xd.shape[1] != self.cols:
            raise MinqError(_lib.ERR_SHAPE, f"matmul input must be [batch, {self.cols}]")
        return self.matmul_device(xd.contiguous()).cpu().numpy()


def matvec_f32(w, x) -> np.ndarray:
    """tensor.rs:181 — dense f32 matvec on the GPU."""
    torch = _torch()
    wd = _dev_tensor(w, torch.float32)
    xd = _dev_tensor(x, torch.float32).reshape(-1)
    y = torch.empty(wd.shape[0], dtype=torch.float32, device="cuda")
    check(lib().minq_matvec_f32(_ptr(wd), wd.shape[0], wd.shape[1], _ptr(xd), xd.numel(),
                                _ptr(y), _stream_ptr()))
    return y.cpu().numpy()


def _to_cconfig(cfg: ModelConfig) -> _lib.Config:
    c = _lib.Config()
    for k in ("hidden_size", "intermediate_size", "n_layers", "n_heads", "n_kv_heads",
              "head_dim", "vocab_size", "max_seq_len"):
        setattr(c, k, int(getattr(cfg, k)))
    c.rope_theta = float(cfg.rope_theta)
    c.rms_norm_eps = float(cfg.rms_norm_eps)
    c.has_qkv_bias = 1 if cfg.has_qkv_bias else 0
    c.dtype = {"f32": TAG_F32, "q8_0": TAG_Q8_0, "q4_0": TAG_Q4_0}.get(cfg.dtype, TAG_F32)
    return c


def _from_cconfig(c: _lib.Config) -> ModelConfig:
    return ModelConfig(
        hidden_size=c.hidden_size, intermediate_size=c.intermediate_size, n_layers=c.n_layers,
        n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim,
        vocab_size=c.vocab_size, max_seq_len=c.max_seq_len,
        rope_theta=float(np.float32(c.rope_theta)), rms_norm_eps=float(np.float32(c.rms_norm_eps)),
        has_qkv_bias=bool(c.has_qkv_bias),
        dtype={TAG_F32: "f32", TAG_Q8_0: "q8_0", TAG_Q4_0: "q4_0"}[c.dtype])


class Model:
    """model.rs:88-98 — weights resident on the GPU."""

    def __init__(self, handle: C.c_void_p):
        self._h = handle
        c = _lib.Config()
        check(lib().minq_model_config(self._h, C.byref(c)))
        self.config = _from_cconfig(c)

    @classmethod
    def load_minq(cls, path) -> "Model":
        """model.rs:711 — parse a .minq file and upload it."""
        h = C.c_void_p()
        check(lib().minq_model_load(str(path).encode(), C.byref(h)))
        return cls(h)

    @classmethod
    def from_tensors(cls, config: ModelConfig, tensors: Iterable) -> "Model":
        """assemble (model.rs:522) from (name, tag, shape, data) records; data
        may be host numpy arrays or CUDA torch tensors."""
        h = C.c_void_p()
        cfg = _to_cconfig(config)
        check(lib().minq_model_new(C.byref(cfg), C.byref(h)))
        try:
            torch = None
            for name, tag, shape, data in tensors:
                shp = (C.c_uint64 * max(len(shape), 1))(*[int(d) for d in shape])
                on_dev = 0
                if hasattr(data, "data_ptr"):
                    torch = torch or _torch()
                    data = data.contiguous()
                    ptr, nbytes = C.c_void_p(data.data_ptr()), data.numel() * data.element_size()
                    on_dev = 1 if data.is_cuda else 0
                    if on_dev:
                        torch.cuda.current_stream().synchronize()
                else:
                    data = np.ascontiguousarray(data)
                    ptr, nbytes = C.c_void_p(data.ctypes.data), data.nbytes
                check(lib().minq_model_add_tensor(h, name.encode(), int(tag), len(shape), shp,
                                                  ptr, nbytes, on_dev))
            check(lib().minq_model_finish(h))
        except Exception:
            lib().minq_model_free(h)
            raise
        return cls(h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and not sys.is_finalizing():  # at interpreter exit the process frees it
            lib().minq_model_free(h)
            self._h = None

    @property
    def weight_bytes(self) -> int:
        v = C.c_uint64()
        check(lib().minq_model_weight_bytes(self._h, C.byref(v)))
        return int(v.value)

    @property
    def stream(self) -> int:
        return lib().minq_model_stream(self._h) or 0

    def new_cache(self, batch: int = 1, max_seq: int = 0) -> "KVCache":
        return KVCache(self, batch, max_seq)

    def forward(self, tokens, cache: "KVCache") -> np.ndarray:
        """model.rs:254 — run tokens, append to the cache, return the last
        token's logits (host)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        check(lib().minq_forward(self._h, cache._h, toks.ctypes.data_as(C.c_void_p), toks.size,
                                 out.ctypes.data_as(C.c_void_p), None))
        return out

    def forward_argmax(self, tokens, cache: "KVCache", logits: bool = False):
        """forward + greedy pick computed on the GPU; returns the token (and the
        logits when asked)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        am = np.zeros(1, dtype=np.uint32)
        out = np.empty(self.config.vocab_size, dtype=np.float32) if logits else None
        check(lib().minq_forward(self._h, cache._h, toks.ctypes.data_as(C.c_void_p), toks.size,
                                 out.ctypes.data_as(C.c_void_p) if logits else None,
                                 am.ctypes.data_as(C.c_void_p)))
        return (int(am[0]), out) if logits else int(am[0])

    def set_graphs(self, enabled: bool) -> None:
        """Replay decode steps as captured CUDA graphs (default) or launch eagerly."""
        check(lib().minq_model_set_graphs(self._h, 1 if enabled else 0))

    def decode_steps(self, cache: "KVCache", n: int, d_tokens_out: int | None = None) -> None:
        """Greedy continuation on the device: n steps, each fed by the previous
        step's argmax; no host synchronisation."""
        check(lib().minq_decode_steps(self._h, cache._h, n,
                                      C.c_void_p(d_tokens_out) if d_tokens_out else None))

    def forward_full_states(self, tokens) -> np.ndarray:
        """Model::forward_full_states (model.rs:337-424): [n, hidden] f32 hidden
        states after the last decoder layer, before the final RMSNorm; one
        causal sweep, no cache kept."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        out = np.empty((t.size, self.config.hidden_size), dtype=np.float32)
        check(lib().minq_forward_full_states(self._h, t.ctypes.data_as(C.c_void_p), t.size,
                                             out.ctypes.data_as(C.c_void_p)))
        return out

    def tp_init(self, rank: int, world: int, unique_id: bytes) -> None:
        """Keep this rank's share of a tensor-parallel split over `world` GPUs and
        join the NCCL communicator named by `unique_id` (tp_unique_id()); every
        rank then calls forward / decode_steps with the same tokens."""
        buf = C.create_string_buffer(bytes(unique_id), 128)
        check(lib().minq_tp_init(self._h, rank, world, buf))

    def forward_batch(self, tokens, cache: "KVCache", logits: bool = True):
        """One batched step: tokens[b] (one per sequence of a batch cache) through
        Model::forward_token (model.rs:273-318) at the cache's position. Returns
        (argmax [batch], logits [batch, vocab] or None), host arrays."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        am = np.zeros(toks.size, dtype=np.uint32)
        out = np.empty((toks.size, self.config.vocab_size), dtype=np.float32) if logits else None
        check(lib().minq_forward_batch(self._h, cache._h, toks.ctypes.data_as(C.c_void_p),
                                       toks.size,
                                       out.ctypes.data_as(C.c_void_p) if logits else None,
                                       am.ctypes.data_as(C.c_void_p)))
        return am, out

    def prefill_batch(self, prompts, cache: "KVCache", logits: bool = True):
        """The prompts of a batch cache: prompts[b] (equal lengths n, one row
        per sequence) through Model::forward (model.rs:254-270) per sequence,
        all but the last tokens in chunks of 64 on the tensor cores, the last
        tokens as one batched step. Returns (argmax [batch], logits [batch,
        vocab] or None) of that step."""
        toks = np.ascontiguousarray(np.asarray(prompts, dtype=np.uint32))
        if toks.ndim != 2:
            raise ValueError("prompts: one row of token ids per sequence")
        B, n = toks.shape
        am = np.zeros(B, dtype=np.uint32)
        out = np.empty((B, self.config.vocab_size), dtype=np.float32) if logits else None
        check(lib().minq_prefill_batch(self._h, cache._h, toks.ctypes.data_as(C.c_void_p), n,
                                       out.ctypes.data_as(C.c_void_p) if logits else None,
                                       am.ctypes.data_as(C.c_void_p)))
        return am, out

    def forward_batch_steps(self, cache: "KVCache", n: int, d_tokens_out: int | None = None):
        """Greedy continuation of a batch cache on the device: n batched steps,
        every sequence fed its previous argmax; no host synchronisation."""
        check(lib().minq_forward_batch_device(self._h, cache._h, n,
                                              C.c_void_p(d_tokens_out) if d_tokens_out else None))

    def forward_device(self, d_tokens, n: int, cache: "KVCache", d_logits=None, d_argmax=None):
        """Device-resident variant (no host synchronisation) on the model's stream."""
        check(lib().minq_forward_device(self._h, cache._h, C.c_void_p(d_tokens), n,
                                        C.c_void_p(d_logits) if d_logits else None,
                                        C.c_void_p(d_argmax) if d_argmax else None))


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Model.tp_init."""
    buf = C.create_string_buffer(128)
    check(lib().minq_tp_unique_id(buf))
    return buf.raw


class KVCache:
    """model.rs:110-131, preallocated in HBM ([batch][n_kv][max_seq][hd] per layer)."""

    def __init__(self, model: Model, batch: int = 1, max_seq: int = 0):
        self.model = model
        self._h = C.c_void_p()
        check(lib().minq_cache_new(model._h, batch, max_seq, C.byref(self._h)))

    def write_device(self, layer: int, start: int, k_ptr: int, v_ptr: int, n: int) -> None:
        """Pre-fill positions [start, start+n) of one layer from device memory
        ([n, n_kv*head_dim] f32 each, this rank's kv heads)."""
        check(lib().minq_cache_write_device(self._h, layer, start, n, C.c_void_p(k_ptr),
                                            C.c_void_p(v_ptr)))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and not sys.is_finalizing():
            lib().minq_cache_free(h)
            self._h = None

    @property
    def len(self) -> int:
        v = C.c_size_t()
        check(lib().minq_cache_len(self._h, C.byref(v)))
        return int(v.value)

    def reset(self) -> None:
        check(lib().minq_cache_reset(self._h))

    def set_len(self, n: int) -> None:
        check(lib().minq_cache_set_len(self._h, n))

    def write(self, layer: int, start: int, k: np.ndarray, v: np.ndarray) -> None:
        """Write positions [start, start+n) of `layer` from [n, n_kv*hd] arrays."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        check(lib().minq_cache_write(self._h, layer, start, k.shape[0],
                                     k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p)))

    def read(self, layer: int, start: int = 0, n: int | None = None):
        cfg = self.model.config
        n = self.len - start if n is None else n
        kvd = cfg.n_kv_heads * cfg.head_dim
        k = np.zeros((n, kvd), dtype=np.float32)
        v = np.zeros((n, kvd), dtype=np.float32)
        check(lib().minq_cache_read(self._h, layer, start, n, k.ctypes.data_as(C.c_void_p),
                                    v.ctypes.data_as(C.c_void_p)))
        return k, v


def eval_ppl(model: "Model", tokens, context: int,
             on_window: Callable[[int, int, float], None] | None = None) -> "PplResult":
    """eval_ppl (ppl.rs:44-103): non-overlapping windows of `context` tokens,
    each swept causally on the GPU; position t in 1 .. len - 2 of a window
    scores the next token by log-sum-exp (f64); `on_window(done, total,
    cumulative_ppl)` after each window. Returns PplResult (total_tokens,
    scored_positions, mean_nll, ppl). An exception raised by on_window is
    re-raised after the call."""
    t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
    raised = []

    def cb(done, total, ppl, _user):
        if on_window is not None and not raised:
            try:
                on_window(int(done), int(total), float(ppl))
            except BaseException as e:  # re-raised after the C call returns
                raised.append(e)

    ccb = _lib.PPL_WINDOW_CB(cb)
    res = PplResult()
    st = lib().minq_eval_ppl(model._h, t.ctypes.data_as(C.c_void_p), t.size, int(context), ccb,
                             None, C.byref(res))
    if raised:
        raise raised[0]
    check(st)
    return res


class Sampler:
    """Sampler (sampler.rs:20-109): temperature (<= 0: greedy), top_k (0: off),
    top_p (>= 1: off) and the StdRng seed. Greedy samplers take the argmax;
    the others draw on the GPU (minq_sampler_*), with the RNG state in device
    memory, created on the current device at the first draw."""

    def __init__(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                 seed: int = 0):
        self.temperature, self.top_k, self.top_p, self.seed = temperature, top_k, top_p, seed
        self._h = None

    @classmethod
    def greedy(cls) -> "Sampler":
        return cls(0.0, 0, 1.0, 0)

    @property
    def is_greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1

    def _handle(self):
        if self._h is None:
            h = C.c_void_p()
            check(lib().minq_sampler_new(float(self.temperature), int(self.top_k),
                                         float(self.top_p), int(self.seed), C.byref(h)))
            self._h = h
        return self._h

    def __del__(self):
        if getattr(self, "_h", None) is not None:
            lib().minq_sampler_free(self._h)
            self._h = None

    def sample(self, logits) -> int:
        """Sampler::sample on host logits (drawn on the GPU)."""
        x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))
        out = np.zeros(1, dtype=np.uint32)
        check(lib().minq_sampler_sample(self._handle(), x.ctypes.data_as(C.c_void_p), x.size,
                                        out.ctypes.data_as(C.c_void_p)))
        return int(out[0])

    def sample_device(self, logits, out) -> None:
        """Sampler::sample on a CUDA f32 tensor into a CUDA int32 tensor of one
        element, on torch's current stream (no host synchronisation)."""
        check(lib().minq_sampler_sample_device(self._handle(), _ptr(logits), logits.numel(),
                                               _ptr(out), _stream_ptr()))

    def rng_u32(self, n: int) -> np.ndarray:
        """The next n raw StdRng outputs (diagnostic; advances the state)."""
        out = np.zeros(n, dtype=np.uint32)
        check(lib().minq_sampler_rng_u32(self._handle(), n, out.ctypes.data_as(C.c_void_p)))
        return out


class Engine:
    """engine.rs:30-88."""

    def __init__(self, model: Model, sampler: Sampler):
        self.model, self.sampler = model, sampler
        self.stop_tokens: list[int] = []

    def generate(self, prompt, max_tokens: int,
                 on_token: Callable[[int], None] | None = None) -> GenStats:
        prompt = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32).reshape(-1))
        stop = np.ascontiguousarray(np.asarray(self.stop_tokens, dtype=np.uint32))
        err: list[BaseException] = []

        def cb(tok, _user):
            if on_token is None:
                return 0
            try:
                on_token(int(tok))
                return 0
            except BaseException as e:  # engine.rs:73: callback errors abort generation
                err.append(e)
                return 1

        ccb = _lib.TOKEN_CB(cb)
        stats = GenStats()
        stop_p = stop.ctypes.data_as(C.c_void_p) if stop.size else None
        if self.sampler.is_greedy:
            st = lib().minq_generate(self.model._h, prompt.ctypes.data_as(C.c_void_p),
                                     prompt.size, max_tokens, stop_p, stop.size, ccb, None, None,
                                     C.byref(stats))
        else:  # tokens drawn on the GPU from each step's logits
            st = lib().minq_generate_sampled(self.model._h, self.sampler._handle(),
                                             prompt.ctypes.data_as(C.c_void_p), prompt.size,
                                             max_tokens, stop_p, stop.size, ccb, None, None,
                                             C.byref(stats))
        if err:
            raise err[0]
        check(st)
        return stats
