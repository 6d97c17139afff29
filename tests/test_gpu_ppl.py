"""The full-sequence sweep (minq_forward_full_states, model.rs:337-424) and
perplexity evaluation (minq_eval_ppl, ppl.rs:44-103) against the CPU oracle.

Tolerances: hidden states max-abs <= 1e-3 x max(1, |ref|) and logits < 1e-3
as in test_gpu_model.py (model.rs:932-940). The negative log-likelihood is
1-Lipschitz in each of the log-sum-exp and the target logit, so a logit
error of e moves a position's nll by at most 2e: mean_nll within 2e-3, ppl
within a relative 2e-3. Position counts, window counts and the
out-of-range-token error after the first window's report are exact."""
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
    ("q4_qwen3_hd128_tied", "q4_0", 512, 768, 8, 2, 128, 300, True, False, True),
    ("q8_qwen2_bias_tied", "q8_0", 256, 512, 8, 2, 64, 257, False, True, True),
    ("q4_llama_untied", "q4_0", 256, 512, 4, 4, 64, 200, False, False, False),
]


def _pair(mq, orc, case, max_seq=256):
    name, dtype, H, I, nh, nkv, hd, V, qkn, bias, tied = case
    cfg = ModelConfig(H, I, 2, nh, nkv, hd, V, max_seq, 1e6, 1e-6, bias, dtype)
    recs = _records(cfg, dtype, orc, 41, qkn, bias, tied)
    model = mq.Model.from_tensors(cfg, recs)
    om = orc.Model.from_tensors(_cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    return cfg, model, om


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_full_states_match_oracle(mq, orc, case):
    cfg, model, om = _pair(mq, orc, case)
    rng = np.random.default_rng(2)
    for n in (1, 5, 64, 65, 150):  # one position, inside a chunk, chunk boundaries
        toks = rng.integers(0, cfg.vocab_size, n)
        got = model.forward_full_states(toks)
        ref = om.forward_full_states(toks)
        assert got.shape == (n, cfg.hidden_size)
        assert np.abs(got - ref).max() <= 1e-3 * max(1.0, float(np.abs(ref).max())), n
    # the sweep's last state gives the cached forward's logits (model.rs:882)
    toks = rng.integers(0, cfg.vocab_size, 70)
    full = om.forward_full(toks)
    _, logits = model.forward_argmax(toks, model.new_cache(), logits=True)
    assert np.abs(logits - full).max() < 1e-3


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("n,context", [(40, 16), (33, 16), (200, 150), (130, 65), (9, 3)])
def test_eval_ppl_matches_oracle(mq, orc, case, n, context):
    cfg, model, om = _pair(mq, orc, case)
    toks = np.random.default_rng(n + 7 * context).integers(0, cfg.vocab_size, n)
    seen = []
    r = mq.eval_ppl(model, toks, context, lambda d, t, p: seen.append((d, t, p)))
    ref = om.eval_ppl(toks, context)
    assert r.total_tokens == n and r.scored_positions == ref["scored_positions"]
    assert abs(r.mean_nll - ref["mean_nll"]) <= 2e-3
    assert abs(r.ppl / ref["ppl"] - 1.0) <= 2.1e-3
    nw = -(-n // context)
    assert [(d, t) for d, t, _ in seen] == [(i + 1, nw) for i in range(nw)]
    got_w = np.array([p for _, _, p in seen])
    assert np.all(np.abs(got_w / ref["windows"] - 1.0) <= 2.1e-3)


def test_eval_ppl_errors(mq, orc):
    from minq_b200._lib import MinqError
    cfg, model, om = _pair(mq, orc, CASES[2], max_seq=64)
    good = list(range(1, 41))
    with pytest.raises(MinqError, match="at least 3 tokens"):
        mq.eval_ppl(model, [1, 2], 16)
    with pytest.raises(MinqError, match="context must be >= 3"):
        mq.eval_ppl(model, good, 2)
    with pytest.raises(MinqError, match="exceeds max_seq_len"):
        mq.eval_ppl(model, good, 65)
    with pytest.raises(MinqError, match="empty token sequence"):
        model.forward_full_states([])
    with pytest.raises(MinqError, match="exceeds max_seq_len"):
        model.forward_full_states(list(range(65)))
    # an out-of-range token in the second window: the first window is reported
    seen = []
    bad = good[:20] + [cfg.vocab_size] + good[21:]
    with pytest.raises(MinqError, match="out of bounds"):
        mq.eval_ppl(model, bad, 16, lambda d, t, p: seen.append(d))
    assert seen == [1]
    # the library still serves after the errors
    r = mq.eval_ppl(model, good, 16)
    assert r.scored_positions == om.eval_ppl(good, 16)["scored_positions"]


def test_eval_ppl_growing_inputs_reuse_one_token_buffer(mq, orc):
    """Inputs past the staged-token buffer's first capacity (4096 ids) grow it
    in place: the old buffer is released, later shorter and longer inputs
    still score like the oracle."""
    cfg, model, om = _pair(mq, orc, CASES[1])
    rng = np.random.default_rng(11)
    for n in (5000, 3000, 9000, 9001):
        toks = rng.integers(0, cfg.vocab_size, n)
        r = mq.eval_ppl(model, toks, 16)
        ref = om.eval_ppl(toks, 16)
        assert r.total_tokens == n and r.scored_positions == ref["scored_positions"]
        assert abs(r.mean_nll - ref["mean_nll"]) <= 2e-3, n
