"""Seeded synthetic models of the benchmark shapes (random-init weights).

There is no network for checkpoints, so models are drawn the way the
benchmark configurations specify: every weight matrix and bias N(0, 0.02)
in f32, norm gains 1.0, then quantized with the `minq quantize` selection
rule (main.rs:343-346: 2-D `.weight` tensors except the embedding) and
emitted in sorted name order (main.rs:303). `random_model` mirrors
Model::random (model.rs:429-474): uniform +-1/sqrt(fan_in) dense f32 weights
with an untied f32 lm_head, for the reference's small test configurations.

Generation uses torch's seeded generator on the requested device (CUDA by
default, so multi-GB models are drawn in seconds); the quantizer is a
parameter and defaults to the GPU quantizer of libminq_cuda.so.
"""
from __future__ import annotations

import zlib
from dataclasses import replace
from typing import Callable, Iterator

import numpy as np

from .minq_format import ModelConfig, TAG_F32, DTYPE_TAGS, quantize_tensor_rule

# Architecture shapes of the benchmark configurations.
QWEN2_0_5B = ModelConfig(hidden_size=896, intermediate_size=4864, n_layers=24, n_heads=14,
                         n_kv_heads=2, head_dim=64, vocab_size=151936, max_seq_len=4096,
                         rope_theta=1e6, rms_norm_eps=1e-6, has_qkv_bias=True, dtype="q8_0")
QWEN3_4B = ModelConfig(hidden_size=2560, intermediate_size=9728, n_layers=36, n_heads=32,
                       n_kv_heads=8, head_dim=128, vocab_size=151936, max_seq_len=4096,
                       rope_theta=1e6, rms_norm_eps=1e-6, has_qkv_bias=False, dtype="q4_0")
LLAMA3_8B = ModelConfig(hidden_size=4096, intermediate_size=14336, n_layers=32, n_heads=32,
                        n_kv_heads=8, head_dim=128, vocab_size=128256, max_seq_len=4096,
                        rope_theta=5e5, rms_norm_eps=1e-5, has_qkv_bias=False, dtype="q4_0")

ARCH = {
    # name: (config, qk_norm, tied)
    "qwen2-0.5b": (QWEN2_0_5B, False, True),
    "qwen3-4b": (QWEN3_4B, True, True),
    "llama3-8b": (LLAMA3_8B, False, False),
}


def tensor_names(cfg: ModelConfig, qk_norm: bool, tied: bool) -> list[tuple[str, list[int]]]:
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qd, kvd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    out = [("model.embed_tokens.weight", [cfg.vocab_size, H])]
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}"
        out += [(f"{p}.input_layernorm.weight", [H]),
                (f"{p}.self_attn.q_proj.weight", [qd, H]),
                (f"{p}.self_attn.k_proj.weight", [kvd, H]),
                (f"{p}.self_attn.v_proj.weight", [kvd, H]),
                (f"{p}.self_attn.o_proj.weight", [H, qd])]
        if cfg.has_qkv_bias:
            out += [(f"{p}.self_attn.q_proj.bias", [qd]), (f"{p}.self_attn.k_proj.bias", [kvd]),
                    (f"{p}.self_attn.v_proj.bias", [kvd])]
        if qk_norm:
            out += [(f"{p}.self_attn.q_norm.weight", [hd]), (f"{p}.self_attn.k_norm.weight", [hd])]
        out += [(f"{p}.post_attention_layernorm.weight", [H]),
                (f"{p}.mlp.gate_proj.weight", [I, H]), (f"{p}.mlp.up_proj.weight", [I, H]),
                (f"{p}.mlp.down_proj.weight", [H, I])]
    out.append(("model.norm.weight", [H]))
    if not tied:
        out.append(("lm_head.weight", [cfg.vocab_size, H]))
    return sorted(out)


def _is_gain(name: str) -> bool:
    return name.endswith("norm.weight")


def _gpu_quantize(tag: int, x):
    from .api import quantize_device
    return quantize_device(tag, x)


def synth_records(cfg: ModelConfig, seed: int, qk_norm: bool, tied: bool, device: str = "cuda",
                  quantize: Callable | None = None, std: float = 0.02) -> Iterator[tuple]:
    """Yield (name, tag, shape, data) records of a seeded N(0, std) model.

    `data` is a torch tensor on `device` (f32 values, or uint8 blocks for
    quantized weights). Each tensor draws from its own generator seeded by
    (seed, crc32(name)), so any subset is reproducible."""
    import torch
    quantize = quantize or _gpu_quantize
    qtag = DTYPE_TAGS[cfg.dtype]
    for name, shape in tensor_names(cfg, qk_norm, tied):
        if _is_gain(name):
            t = torch.ones(shape, dtype=torch.float32, device=device)
        else:
            g = torch.Generator(device=device)
            g.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
            t = torch.randn(shape, generator=g, dtype=torch.float32, device=device) * std
        if qtag != TAG_F32 and quantize_tensor_rule(name, shape):
            yield name, qtag, shape, quantize(qtag, t)
        else:
            yield name, TAG_F32, shape, t


def random_model_records(cfg: ModelConfig, seed: int, qk_norm: bool = False,
                         with_bias: bool = False) -> Iterator[tuple]:
    """Model::random (model.rs:429-474): uniform [-1/sqrt(fan_in), +1/sqrt(fan_in))
    dense f32 weights, gains 1.0, untied f32 lm_head; optional Qwen3 q/k gains
    in [0.5, 1.5) (model.rs:868-879) and biases. Host numpy arrays."""
    rng = np.random.default_rng(seed)
    cfg = replace(cfg, dtype="f32", has_qkv_bias=with_bias)
    for name, shape in tensor_names(cfg, qk_norm, tied=False):
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            data = (0.5 + rng.random(shape)).astype(np.float32)
        elif _is_gain(name):
            data = np.ones(shape, dtype=np.float32)
        elif name.endswith(".bias"):
            data = ((rng.random(shape) - 0.5) * 0.2).astype(np.float32)
        else:
            scale = 1.0 / np.sqrt(np.float32(shape[-1]))
            data = ((rng.random(shape, dtype=np.float32) - 0.5) * 2.0 * scale).astype(np.float32)
        yield name, TAG_F32, shape, data


def to_host(records) -> list[tuple]:
    """Materialise records as host numpy arrays (for the .minq writer / oracle)."""
    out = []
    for name, tag, shape, data in records:
        if hasattr(data, "detach"):
            data = data.detach().cpu().numpy()
        out.append((name, tag, list(shape), np.ascontiguousarray(data)))
    return out
