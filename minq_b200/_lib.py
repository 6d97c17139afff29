"""ctypes binding of libminq_cuda.so (the C ABI of include/minq_cuda.h).

There is no fallback: if the shared library is missing or cannot be loaded,
importing this module raises, and every compute call without a CUDA device
returns MINQ_ERR_CUDA, raised here as MinqError.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libminq_cuda.so")

# minq_status (error.rs:5-28 variants + device failures)
OK, ERR_IO, ERR_SHAPE, ERR_FORMAT, ERR_MODEL, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_ARG = range(9)
STATUS_NAMES = {
    ERR_IO: "Io", ERR_SHAPE: "Shape", ERR_FORMAT: "Format", ERR_MODEL: "Model",
    ERR_CUDA: "Cuda", ERR_NCCL: "Nccl", ERR_TIMEOUT: "Timeout", ERR_ARG: "Arg",
}

F32, Q8_0, Q4_0 = 0, 1, 2


class MinqError(RuntimeError):
    """MinqError (error.rs:5-28) raised from a non-zero minq_status."""

    def __init__(self, status: int, msg: str):
        self.status = status
        self.kind = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.kind} error: {msg}")


class Config(C.Structure):
    """minq_config == ModelConfig (model.rs:29-45)."""

    _fields_ = [
        ("hidden_size", C.c_uint64), ("intermediate_size", C.c_uint64),
        ("n_layers", C.c_uint64), ("n_heads", C.c_uint64), ("n_kv_heads", C.c_uint64),
        ("head_dim", C.c_uint64), ("vocab_size", C.c_uint64), ("max_seq_len", C.c_uint64),
        ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
        ("has_qkv_bias", C.c_int32), ("dtype", C.c_int32),
    ]


class GenStats(C.Structure):
    """minq_gen_stats == GenStats (engine.rs:11-27)."""

    _fields_ = [("prompt_tokens", C.c_uint64), ("gen_tokens", C.c_uint64),
                ("prefill_secs", C.c_double), ("decode_secs", C.c_double)]

    def prefill_tokens_per_sec(self) -> float:  # engine.rs:20-22
        return self.prompt_tokens / max(self.prefill_secs, 1e-9)

    def decode_tokens_per_sec(self) -> float:  # engine.rs:24-26
        return self.gen_tokens / max(self.decode_secs, 1e-9)


class PplResult(C.Structure):
    """minq_ppl_result == PplResult (ppl.rs:16-27)."""

    _fields_ = [("total_tokens", C.c_uint64), ("scored_positions", C.c_uint64),
                ("mean_nll", C.c_double), ("ppl", C.c_double)]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_uint32, C.c_void_p)
PPL_WINDOW_CB = C.CFUNCTYPE(None, C.c_size_t, C.c_size_t, C.c_double, C.c_void_p)

P, S, I, U64P = C.c_void_p, C.c_size_t, C.c_int, C.POINTER(C.c_uint64)

# Every exported symbol with its signature; the CPU test suite checks that the
# library exports exactly these names (and that include/minq_cuda.h declares them).
SIGNATURES = {
    "minq_last_error": (C.c_char_p, []),
    "minq_abi_version": (I, []),
    "minq_kernel_launches": (C.c_uint64, []),
    "minq_device_status": (I, []),
    "minq_kernel_timer_start": (I, [C.c_char_p]),
    "minq_kernel_timer_stop": (I, [U64P, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "minq_quantize": (I, [I, P, S, P, P]),
    "minq_dequantize": (I, [I, P, S, P, S, P]),
    "minq_qmatvec": (I, [I, P, S, S, P, S, P, P]),
    "minq_qmatmul_workspace_bytes": (S, [S, S, S]),
    "minq_qmatmul": (I, [I, P, S, S, P, S, P, P, S, P]),
    "minq_matvec_f32": (I, [P, S, S, P, S, P, P]),
    "minq_argmax": (I, [P, S, P, P]),
    "minq_attn_workspace_bytes": (S, [S, S, S]),
    "minq_attn_decode": (I, [P, P, P, P, P, C.c_float, P, P, S, S, S, S, S, P, P, S, S, S, P, P,
                             S, P]),
    "minq_attend": (I, [P, P, P, S, S, S, S, P, P, S, P]),
    "minq_attend_static": (I, [P, P, P, S, S, S, S, P, P]),
    "minq_attn_prefill_workspace_bytes": (S, [S, S, S, S]),
    "minq_attend_prefill": (I, [P, P, P, S, S, S, S, S, S, P, P, S, P]),
    "minq_attend_static_status": (I, []),
    "minq_model_load": (I, [C.c_char_p, C.POINTER(P)]),
    "minq_model_new": (I, [C.POINTER(Config), C.POINTER(P)]),
    "minq_model_add_tensor": (I, [P, C.c_char_p, I, S, U64P, P, S, I]),
    "minq_model_finish": (I, [P]),
    "minq_model_config": (I, [P, C.POINTER(Config)]),
    "minq_model_weight_bytes": (I, [P, U64P]),
    "minq_model_free": (None, [P]),
    "minq_model_stream": (P, [P]),
    "minq_cache_new": (I, [P, S, S, C.POINTER(P)]),
    "minq_cache_reset": (I, [P]),
    "minq_cache_len": (I, [P, C.POINTER(C.c_size_t)]),
    "minq_cache_write": (I, [P, S, S, S, P, P]),
    "minq_cache_read": (I, [P, S, S, S, P, P]),
    "minq_cache_set_len": (I, [P, S]),
    "minq_cache_free": (None, [P]),
    "minq_forward": (I, [P, P, P, S, P, P]),
    "minq_forward_device": (I, [P, P, P, S, P, P]),
    "minq_decode_steps": (I, [P, P, S, P]),
    "minq_forward_batch": (I, [P, P, P, S, P, P]),
    "minq_prefill_batch": (I, [P, P, P, S, P, P]),
    "minq_tp_unique_id": (I, [P]),
    "minq_cache_write_device": (I, [P, S, S, S, P, P]),
    "minq_tp_init": (I, [P, C.c_int, C.c_int, P]),
    "minq_forward_batch_device": (I, [P, P, S, P]),
    "minq_model_set_graphs": (I, [P, I]),
    "minq_generate": (I, [P, P, S, S, P, S, TOKEN_CB, P, P, C.POINTER(GenStats)]),
    "minq_forward_full_states": (I, [P, P, S, P]),
    "minq_eval_ppl": (I, [P, P, S, S, PPL_WINDOW_CB, P, C.POINTER(PplResult)]),
    "minq_sampler_new": (I, [C.c_float, S, C.c_float, C.c_uint64, C.POINTER(C.c_void_p)]),
    "minq_sampler_free": (None, [P]),
    "minq_sampler_sample_device": (I, [P, P, S, P, P]),
    "minq_sampler_sample": (I, [P, P, S, P]),
    "minq_sampler_rng_u32": (I, [P, S, P]),
    "minq_generate_sampled": (I, [P, P, P, S, S, P, S, TOKEN_CB, P, P, C.POINTER(GenStats)]),
    "minq_debug_inject_timeout": (I, [P, I]),
}

_lib = None


def lib():
    """Load libminq_cuda.so (raises OSError if it is missing: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python -m minq_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        raise MinqError(status, lib().minq_last_error().decode(errors="replace"))
