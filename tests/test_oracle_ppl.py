"""Perplexity evaluation (ppl.rs:44-103) in the oracle, pinned two ways:

* the reference's own ppl tests (ppl.rs:121-160) on its tiny f32 shape
  (model.rs:723-738) with the same token sequence ((i * 37 + 11) % 128):
  scored-position counts per window layout (40 tokens / context 16 -> 34;
  33 / 16 -> 28 with a 1-token tail), a finite ppl >= 1 equal to
  exp(mean_nll), and ppl within a factor 2 across context sizes;
* a numpy restatement built from the oracle's forward_full_states, rmsnorm
  and f32 lm_head: windows, positions 1 .. len - 2, log-sum-exp in f64
  (ppl.rs:30-35), the per-window cumulative ppl that on_window receives.

The reference's Model::random draws from rand's StdRng, which the oracle does
not restate; the weights here come from the package's seeded generator, so
the pins are the reference's laws, not its numbers."""
import numpy as np
import pytest

from minq_b200 import synth
from minq_b200.minq_format import ModelConfig

TINY = ModelConfig(64, 128, 2, 4, 4, 16, 128, 64, 10000.0, 1e-5, False, "f32")


def _tiny(orc, seed):
    recs = {n: (t, s, d) for n, t, s, d in synth.random_model_records(TINY, seed)}
    cfg = {k: getattr(TINY, k) for k in TINY.__dataclass_fields__}
    return orc.Model.from_tensors(cfg, recs), recs


def _token_seq(n):
    return [(i * 37 + 11) % 128 for i in range(n)]


def test_ppl_is_finite_and_at_least_one(orc):  # ppl.rs:121-132
    om, _ = _tiny(orc, 5)
    r = om.eval_ppl(_token_seq(40), 16)
    assert r["total_tokens"] == 40
    assert r["scored_positions"] == 14 + 14 + 6
    assert np.isfinite(r["ppl"]) and r["ppl"] >= 1.0
    assert abs(r["ppl"] - np.exp(r["mean_nll"])) < 1e-9


def test_ppl_is_similar_across_context_sizes(orc):  # ppl.rs:134-150
    om, _ = _tiny(orc, 6)
    toks = _token_seq(96)
    p = [om.eval_ppl(toks, c)["ppl"] for c in (16, 32, 64)]
    for a, b in [(p[0], p[1]), (p[1], p[2]), (p[0], p[2])]:
        assert 0.5 <= a / b <= 2.0


def test_ppl_handles_uneven_final_window(orc):  # ppl.rs:152-160
    om, _ = _tiny(orc, 7)
    r = om.eval_ppl(_token_seq(33), 16)
    assert r["scored_positions"] == 14 + 14
    assert np.isfinite(r["ppl"]) and r["ppl"] >= 1.0
    w = r["windows"]  # the 1-token tail scores nothing: its report repeats the second's
    assert len(w) == 3 and np.all(np.isfinite(w)) and w[2] == w[1]


def test_ppl_errors(orc):  # ppl.rs:51-68
    om, _ = _tiny(orc, 1)
    with pytest.raises(orc.OracleError, match="at least 3 tokens"):
        om.eval_ppl([1, 2], 16)
    with pytest.raises(orc.OracleError, match="context must be >= 3"):
        om.eval_ppl(_token_seq(10), 2)
    with pytest.raises(orc.OracleError, match="exceeds max_seq_len"):
        om.eval_ppl(_token_seq(10), 65)


def _numpy_ppl(orc, om, recs, toks, context):
    emb = recs["model.embed_tokens.weight"][2].reshape(TINY.vocab_size, TINY.hidden_size)
    norm = recs["model.norm.weight"][2]
    lm = recs["lm_head.weight"][2].reshape(TINY.vocab_size, TINY.hidden_size) \
        if "lm_head.weight" in recs else emb
    total, count, windows = 0.0, 0, []
    for w0 in range(0, len(toks), context):
        win = toks[w0:w0 + context]
        st = om.forward_full_states(win)
        for t in range(1, len(win) - 1):
            xn = orc.rmsnorm(st[t], norm, TINY.rms_norm_eps)
            logits = orc.matvec_f32(lm, xn)
            mx = np.float32(logits.max())
            lse = float(mx) + np.log(np.sum(np.exp((logits - mx).astype(np.float64))))
            total += lse - float(logits[win[t + 1]])
            count += 1
        windows.append(np.exp(total / count) if count else np.nan)
    return count, total / count, np.array(windows)


@pytest.mark.parametrize("n,context", [(40, 16), (33, 16), (64, 64), (50, 3), (20, 7)])
def test_oracle_ppl_matches_numpy_restatement(orc, n, context):
    om, recs = _tiny(orc, 11)
    toks = list(np.random.default_rng(n * 100 + context).integers(0, 128, n))
    r = om.eval_ppl(toks, context)
    count, mean, windows = _numpy_ppl(orc, om, recs, toks, context)
    assert r["scored_positions"] == count
    assert abs(r["mean_nll"] - mean) <= 1e-12 * max(1.0, abs(mean))
    np.testing.assert_allclose(r["windows"], windows, rtol=1e-12)


def test_oracle_nll_is_log_sum_exp(orc):  # ppl.rs:30-35
    x = np.random.default_rng(3).standard_normal(5000).astype(np.float32) * 4
    mx = np.float32(x.max())
    ref = float(mx) + np.log(np.sum(np.exp((x - mx).astype(np.float64)))) - float(x[123])
    assert abs(orc.nll(x, 123) - ref) <= 1e-12 * abs(ref)
    u = np.zeros(1000, dtype=np.float32)  # uniform logits: nll = ln(V)
    assert abs(orc.nll(u, 7) - np.log(1000.0)) < 1e-12
