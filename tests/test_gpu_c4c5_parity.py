"""Parity on the batched and long-context shapes themselves, against the CPU
oracle (`forward_token`, model.rs:273-318; the greedy loop of engine.rs:52-88).

* Batched (LLaMA-3-8B layer shape in Q4_0: hidden 4096, intermediate 14336,
  32 query / 8 kv heads of 128, untied lm_head, RoPE theta 5e5), a 2-layer cut
  with an 8192-entry vocabulary, 64 sequences: 96-token prompts through
  minq_prefill_batch (one full and one ragged chunk of 64 on the tensor
  cores), then batched greedy steps (tensor-core projections from 2 inputs
  on). Sequences 0, 31 and 63 are checked: their last-prompt logits against
  the oracle's forward of the same prompt, and their greedy continuations
  inside the batch against the oracle's.
* Long context (Qwen3-4B layer shape in Q8_0 with q/k RMSNorm), a 4-layer cut
  with an 8192-entry vocabulary: the K/V cache pre-filled at 32768 positions
  with seeded N(0, 1) values, then greedy tokens on the decode megakernel
  against the oracle decoding from a copy of the same cache.

Tolerances as in test_gpu_model.py: logits max-abs < 1e-3 (model.rs:932-940),
greedy tokens identical.
"""
from dataclasses import replace

import numpy as np
import pytest

from minq_b200 import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _cfg_dict(c):
    return {k: getattr(c, k) for k in c.__dataclass_fields__}


def _pair(mq, orc, arch, cfg, seed):
    """The same seeded model on the GPU (device quantizer) and in the oracle
    (host quantizer; both follow quantize.rs:78-143 bit for bit)."""
    import torch
    from minq_b200.minq_format import quantize_tensor_rule, DTYPE_TAGS
    _, qk_norm, tied = synth.ARCH[arch]
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


def _greedy(orc, om, oc, start, n):
    toks, margins = [], []
    tok = start
    for _ in range(n):
        lg = om.forward([tok], oc)
        tok = int(orc.argmax(lg))
        top2 = np.partition(lg, -2)[-2:]
        toks.append(tok)
        margins.append(float(top2[1] - top2[0]))
    return toks, margins


def _check_greedy(got, want, margins, what):
    first = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    assert first is None, (f"{what}: greedy tokens differ from step {first} "
                           f"(oracle top-2 margin there {margins[first]:.3g})")


def test_c4_shape_batched_prefill_and_steps(mq, orc):
    orc.set_threads(orc.max_threads())
    orc.set_attn_parallel(True)
    B, PROMPT, STEPS = 64, 96, 24
    base = synth.ARCH["llama3-8b"][0]
    cfg = replace(base, n_layers=2, vocab_size=8192, max_seq_len=PROMPT + STEPS + 8)
    try:
        model, om = _pair(mq, orc, "llama3-8b", cfg, 11)
        prompts = np.random.default_rng(29).integers(0, cfg.vocab_size, (B, PROMPT))
        cache = model.new_cache(batch=B)
        am, logits = model.prefill_batch(prompts, cache)
        got = [[int(t)] for t in am]
        for _ in range(STEPS - 1):
            a, _ = model.forward_batch([g[-1] for g in got], cache, logits=False)
            for s in range(B):
                got[s].append(int(a[s]))
        for b in (0, 31, 63):
            oc = om.new_cache()
            ref = om.forward(list(prompts[b]), oc)
            err = float(np.abs(logits[b] - ref).max())
            assert err < 1e-3, (b, err)
            first = int(orc.argmax(ref))
            assert got[b][0] == first, b
            want, margins = _greedy(orc, om, oc, first, STEPS - 1)
            _check_greedy(got[b][1:], want, margins, f"sequence {b}")
    finally:
        orc.set_attn_parallel(False)


def test_c5_shape_32k_history_megakernel_greedy(mq, orc):
    import torch
    from minq_b200 import _lib
    orc.set_threads(orc.max_threads())
    orc.set_attn_parallel(True)
    CTX, GREEDY = 32768, 12
    base = synth.ARCH["qwen3-4b"][0]
    cfg = replace(base, dtype="q8_0", n_layers=4, vocab_size=8192,
                  max_seq_len=CTX + GREEDY + 8)
    try:
        model, om = _pair(mq, orc, "qwen3-4b", cfg, 13)
        cache = model.new_cache()
        kvd = cfg.n_kv_heads * cfg.head_dim
        g = torch.Generator(device="cuda").manual_seed(41)
        for li in range(cfg.n_layers):  # the long-context history (model.rs:103-114)
            k = torch.randn(CTX, kvd, device="cuda", generator=g)
            v = torch.randn(CTX, kvd, device="cuda", generator=g)
            cache.write_device(li, 0, k.data_ptr(), v.data_ptr(), CTX)
            del k, v
        cache.set_len(CTX)
        kall = np.empty((cfg.n_layers, CTX, kvd), np.float32)
        vall = np.empty((cfg.n_layers, CTX, kvd), np.float32)
        for li in range(cfg.n_layers):
            kall[li], vall[li] = cache.read(li, 0, CTX)
        oc = om.new_cache()
        oc.fill(kall, vall)
        del kall, vall
        got = []
        t = 1
        for _ in range(GREEDY):
            t = model.forward_argmax([t], cache)
            got.append(int(t))
        want, margins = _greedy(orc, om, oc, 1, GREEDY)
        _check_greedy(got, want, margins, "32768-position history")
        lib = _lib.lib()
        n0 = lib.minq_kernel_launches()
        model.decode_steps(cache, 1)
        torch.cuda.synchronize()
        assert lib.minq_kernel_launches() - n0 == 1, "the decode megakernel did not run"
    finally:
        orc.set_attn_parallel(False)
