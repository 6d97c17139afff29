"""minq_b200 — B200 (sm_100a) implementation of minq's KV-cached forward path.

The kernels live in libminq_cuda.so (C ABI: include/minq_cuda.h); this
package is the Python host mirror of the reference's Rust API. Importing it
does not load CUDA; the first compute call does, and raises MinqError when
no GPU is present (there is no CPU fallback).
"""
from .minq_format import ModelConfig, read_minq, write_minq  # noqa: F401
from ._lib import MinqError, LIB_PATH  # noqa: F401
from .api import (  # noqa: F401
    BLOCK_SIZE, Engine, GenStats, KVCache, Model, PplResult, QuantDtype, QuantizedTensor, Sampler,
    argmax, dequantize_q4_0, dequantize_q8_0, eval_ppl, matvec_f32, quantize_q4_0, quantize_q8_0,
    tp_unique_id,
)

__version__ = "0.1.0"
