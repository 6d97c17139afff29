"""Chunked prompt prefill (minq_forward with a prompt of two or more tokens:
every token but the last in chunks of 64, the projections batched over the
chunk's tokens on the tensor cores, causal attention per token; the last
token as a decode step) against the CPU oracle and against token-by-token
prefill of the same library (MINQ_CHUNKED_PREFILL=0).

Prompts of 2, 65 (one full chunk + the last token), 150 (chunks of 64, 64,
21) tokens, from an empty cache and after earlier tokens. Tolerances as in
test_gpu_model.py: logits max-abs < 1e-3 (model.rs:932-940), K/V cache
within 1e-4, greedy tokens identical."""
import os

import numpy as np
import pytest

from minq_b200 import synth
from minq_b200.minq_format import ModelConfig, quantize_tensor_rule

pytestmark = pytest.mark.gpu


def _cfg_dict(c):
    return {k: getattr(c, k) for k in c.__dataclass_fields__}


def _records(cfg, dtype, orc, seed, qk_norm, bias, tied):
    dt = 1 if dtype == "q8_0" else 2
    out = []
    for n, t, s, d in synth.random_model_records(cfg, seed, qk_norm=qk_norm, with_bias=bias):
        if tied and n == "lm_head.weight":
            continue
        if quantize_tensor_rule(n, s):
            out.append((n, dt, s, orc.quantize(dt, d)))
        else:
            out.append((n, t, s, d))
    return out


CASES = [
    # name, dtype, hidden, inter, heads, kv heads, head_dim, vocab, qk_norm, bias, tied
    ("q4_qwen3_hd128", "q4_0", 512, 768, 8, 2, 128, 300, True, False, True),
    ("q8_qwen2_bias_hd64", "q8_0", 256, 512, 8, 2, 64, 257, False, True, True),
    ("q4_llama_untied", "q4_0", 256, 512, 4, 4, 64, 200, False, False, False),
]


def _chunked(enabled):
    if enabled:
        os.environ.pop("MINQ_CHUNKED_PREFILL", None)
    else:
        os.environ["MINQ_CHUNKED_PREFILL"] = "0"


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_chunked_prefill_matches_oracle_and_token_by_token(mq, orc, case):
    name, dtype, H, I, nh, nkv, hd, V, qkn, bias, tied = case
    cfg = ModelConfig(H, I, 2, nh, nkv, hd, V, 256, 1e6, 1e-6, bias, dtype)
    recs = _records(cfg, dtype, orc, 31, qkn, bias, tied)
    model = mq.Model.from_tensors(cfg, recs)
    om = orc.Model.from_tensors(_cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    rng = np.random.default_rng(11)
    try:
        for plen, pre in ((2, 0), (65, 0), (150, 0), (70, 9)):
            earlier = list(rng.integers(0, V, pre))
            prompt = list(rng.integers(0, V, plen))
            caches, logits, toks = [], [], []
            for enabled in (True, False):
                _chunked(enabled)
                c = model.new_cache()
                if earlier:
                    model.forward(earlier, c)
                tok, lg = model.forward_argmax(prompt, c, logits=True)
                caches.append(c)
                logits.append(lg)
                toks.append(tok)
            _chunked(True)
            oc = om.new_cache()
            if earlier:
                om.forward(earlier, oc)
            ref = om.forward(prompt, oc)
            assert np.abs(logits[0] - ref).max() < 1e-3, (plen, pre)
            assert np.abs(logits[0] - logits[1]).max() < 1e-3, (plen, pre)
            assert toks[0] == toks[1] == int(orc.argmax(ref))
            for li in range(cfg.n_layers):
                k0, v0 = caches[0].read(li)
                k1, v1 = caches[1].read(li)
                n = pre + plen
                assert np.abs(k0[:n] - k1[:n]).max() < 1e-4, (plen, pre, li)
                assert np.abs(v0[:n] - v1[:n]).max() < 1e-4, (plen, pre, li)
            # greedy continuation from the chunked cache: the oracle's tokens
            got = [toks[0]]
            for _ in range(6):
                got.append(model.forward_argmax([got[-1]], caches[0]))
            want, _ = orc.greedy_generate(om, earlier + prompt, 7)
            assert got == want, (plen, pre)
    finally:
        _chunked(True)
