"""Parity on the Qwen3-4B Q4_0 shape itself (hidden 2560, intermediate 9728,
32 query / 8 kv heads of 128, q/k RMSNorm, tied f32 embedding): a
2048-token prompt through the chunked prefill, then greedy decode on the
decode megakernel, against the CPU oracle (`forward_token`, model.rs:273-318;
the greedy loop of engine.rs:52-88).

* A 4-layer cut with a 8192-entry vocabulary (the oracle computes an lm_head
  row set per prompt token as the reference does, so its cost is linear in
  layers and vocabulary; the K/V cache does not depend on the vocabulary
  size): every layer's 2048-position K/V cache and the last prompt token's
  logits against the oracle's own prefill, then 64 greedy tokens from the
  GPU's cache against the oracle decoding from a copy of it.
* The full 36-layer model with the full 151,936-entry vocabulary: 64 greedy
  tokens decoded by the megakernel after the GPU's 2048-token prefill
  against the oracle decoding from a copy of that cache (the headline
  bench's parity record, as a test).

Tolerances as in test_gpu_model.py: K/V max-abs <= 1e-4 x max(1, max|ref|),
logits max-abs < 1e-3 (model.rs:932-940), greedy tokens identical.
"""
from dataclasses import replace

import numpy as np
import pytest

from minq_b200 import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

PROMPT = 2048
GREEDY = 64


def _cfg_dict(c):
    return {k: getattr(c, k) for k in c.__dataclass_fields__}


def _pair(mq, orc, cfg, seed):
    """The same seeded model on the GPU (device quantizer) and in the oracle
    (host quantizer; both follow quantize.rs:78-143 bit for bit)."""
    import torch
    from minq_b200.minq_format import quantize_tensor_rule, DTYPE_TAGS
    base, qk_norm, tied = synth.ARCH["qwen3-4b"]
    model = mq.Model.from_tensors(cfg, synth.synth_records(cfg, seed, qk_norm, tied))
    torch.cuda.synchronize()
    qtag = DTYPE_TAGS[cfg.dtype]
    tensors = {}
    for name, tag, shape, data in synth.synth_records(cfg, seed, qk_norm, tied,
                                                      quantize=lambda t, x: x):
        host = data.detach().cpu().numpy()
        del data
        if quantize_tensor_rule(name, shape):
            tensors[name] = (qtag, shape, orc.quantize(qtag, host))
        else:
            tensors[name] = (0, shape, host)
    om = orc.Model.from_tensors(_cfg_dict(cfg), tensors)
    del tensors
    torch.cuda.empty_cache()
    return model, om


def _launches_per_step(model, cache):
    import torch
    from minq_b200 import _lib
    lib = _lib.lib()
    n0 = lib.minq_kernel_launches()
    model.decode_steps(cache, 1)
    torch.cuda.synchronize()
    return lib.minq_kernel_launches() - n0


def _greedy_from_copy(orc, om, cache, cfg, start, n):
    """The oracle's greedy continuation from a copy of the GPU cache."""
    kvd = cfg.n_kv_heads * cfg.head_dim
    n_pos = cache.len
    kall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
    vall = np.empty((cfg.n_layers, n_pos, kvd), np.float32)
    for li in range(cfg.n_layers):
        kall[li], vall[li] = cache.read(li, 0, n_pos)
    oc = om.new_cache()
    oc.fill(kall, vall)
    del kall, vall
    toks, margins = [], []
    tok = start
    for _ in range(n):
        lg = om.forward([tok], oc)
        tok = int(orc.argmax(lg))
        top2 = np.partition(lg, -2)[-2:]
        toks.append(tok)
        margins.append(float(top2[1] - top2[0]))
    return toks, margins


def _check_greedy(got, want, margins):
    first = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    assert first is None, (f"greedy tokens differ from step {first} "
                           f"(oracle top-2 margin there {margins[first]:.3g})")


def test_c3_4layer_prefill_cache_logits_and_greedy(mq, orc):
    orc.set_threads(orc.max_threads())
    base = synth.ARCH["qwen3-4b"][0]
    cfg = replace(base, n_layers=4, vocab_size=8192, max_seq_len=PROMPT + GREEDY + 8)
    model, om = _pair(mq, orc, cfg, 5)
    prompt = np.random.default_rng(17).integers(0, cfg.vocab_size, PROMPT).astype(np.uint32)
    cache = model.new_cache()
    tok, logits = model.forward_argmax(prompt, cache, logits=True)
    oc = om.new_cache()
    ref = om.forward(prompt, oc)
    assert cache.len == oc.len == PROMPT
    for li in range(cfg.n_layers):
        k, v = cache.read(li)
        rk, rv = oc.read(li)
        for name, got, want in (("k", k, rk), ("v", v, rv)):
            err = float(np.abs(got - want).max())
            assert err <= 1e-4 * max(1.0, float(np.abs(want).max())), (li, name, err)
    assert float(np.abs(logits - ref).max()) < 1e-3
    assert tok == int(orc.argmax(ref))
    # greedy continuation on the decode megakernel (one launch per token)
    got = []
    t = tok
    for _ in range(GREEDY):
        t = model.forward_argmax([t], cache)
        got.append(int(t))
    # the oracle continues from its own prefill cache (its own K/V throughout)
    want, margins = [], []
    t = tok
    for _ in range(GREEDY):
        lg = om.forward([t], oc)
        t = int(orc.argmax(lg))
        top2 = np.partition(lg, -2)[-2:]
        want.append(t)
        margins.append(float(top2[1] - top2[0]))
    _check_greedy(got, want, margins)
    assert _launches_per_step(model, cache) == 1, "the decode megakernel did not run"


def test_c3_full_prefill_then_megakernel_greedy(mq, orc):
    orc.set_threads(orc.max_threads())
    base = synth.ARCH["qwen3-4b"][0]
    cfg = replace(base, max_seq_len=PROMPT + GREEDY + 8)
    model, om = _pair(mq, orc, cfg, 7)
    prompt = np.random.default_rng(23).integers(0, cfg.vocab_size, PROMPT).astype(np.uint32)
    cache = model.new_cache()
    first = model.forward_argmax(prompt, cache)
    n_pos = cache.len
    want, margins = _greedy_from_copy(orc, om, cache, cfg, first, GREEDY)
    got = []
    t = first
    for _ in range(GREEDY):
        t = model.forward_argmax([t], cache)
        got.append(int(t))
    assert cache.len == n_pos + GREEDY
    _check_greedy(got, want, margins)
    assert _launches_per_step(model, cache) == 1, "the decode megakernel did not run"
