"""GPU model parity: the reference's model/engine tests (model.rs:797-940,
engine.rs:97-139) run on the CUDA path and compared with the CPU oracle, plus
greedy-token identity on the benchmark architectures.

Tolerances: logits max-abs < 1e-3 (the reference's own assert_logits_close,
model.rs:932-940); K/V cache entries within 1e-4 of the oracle's; greedy
token ids identical (first 64 tokens)."""
import numpy as np
import pytest

from minq_b200 import synth
from minq_b200.minq_format import ModelConfig, write_minq

pytestmark = pytest.mark.gpu

F = np.float32


def tiny_config(n_kv, dtype="f32", hidden=64, inter=128):  # model.rs:723
    return ModelConfig(hidden, inter, 2, 4, n_kv, 16, 128, 64, 10000.0, 1e-5, False, dtype)


def qwen3_tiny_config():  # model.rs:850
    return ModelConfig(64, 128, 2, 4, 2, 8, 128, 64, 1e6, 1e-6, False, "f32")


def cfg_dict(c):
    return {k: getattr(c, k) for k in c.__dataclass_fields__}


def quantize_records(records, dt, orc):
    """`minq quantize` on host records, with the oracle's quantizer."""
    from minq_b200.minq_format import quantize_tensor_rule
    out = []
    for n, t, s, d in records:
        if quantize_tensor_rule(n, s):
            out.append((n, dt, s, orc.quantize(dt, d)))
        else:
            out.append((n, t, s, d))
    return out


def both(mq, orc, cfg, records):
    recs = list(records)
    gm = mq.Model.from_tensors(cfg, recs)
    om = orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    return gm, om


def close(a, b, tol=1e-3):
    assert a.shape == b.shape
    d = np.abs(a - b).max()
    assert d < tol, d


@pytest.mark.parametrize("dtype", ["f32", "q8_0", "q4_0"])
def test_kv_cache_matches_full_forward(mq, orc, dtype):  # model.rs:798
    cfg = tiny_config(4, dtype=dtype, hidden=128, inter=256)
    recs = list(synth.random_model_records(cfg, 7))
    if dtype != "f32":
        recs = quantize_records(recs, 1 if dtype == "q8_0" else 2, orc)
    gm, om = both(mq, orc, cfg, recs)
    toks = [5, 11, 23, 97, 3, 42]
    ref = om.forward_full(toks)
    c = gm.new_cache()
    for t in toks:
        last = gm.forward([t], c)
    close(ref, last)
    c = gm.new_cache()
    gm.forward(toks[:4], c)
    close(ref, gm.forward(toks[4:], c))
    # K/V cache (post-RoPE keys) against the oracle's incremental cache
    oc = om.new_cache()
    om.forward(toks, oc)
    for layer in range(cfg.n_layers):
        gk, gv = c.read(layer)
        ok, ov = oc.read(layer)
        assert np.abs(gk - ok).max() < 1e-4 and np.abs(gv - ov).max() < 1e-4


def test_tiny_reference_config_hd16_hidden64(mq, orc):
    cfg = tiny_config(2)
    gm, om = both(mq, orc, cfg, synth.random_model_records(cfg, 3))
    toks = [1, 2, 3, 4, 5, 6, 7]
    close(om.forward_full(toks), gm.forward(toks, gm.new_cache()))


def test_gqa_broadcast_matches_expanded_kv(mq, orc):  # model.rs:819
    cfg = tiny_config(1)
    recs = list(synth.random_model_records(cfg, 42))
    gqa = mq.Model.from_tensors(cfg, recs)
    exp = []
    for n, t, s, d in recs:
        if n.endswith(("k_proj.weight", "v_proj.weight")):
            d = np.concatenate([d] * 4, axis=0)
            s = [s[0] * 4, s[1]]
        exp.append((n, t, s, d))
    mha = mq.Model.from_tensors(tiny_config(4), exp)
    toks = [1, 2, 3, 4, 5]
    close(gqa.forward(toks, gqa.new_cache()), mha.forward(toks, mha.new_cache()))


def test_qwen3_kv_cache_matches_full_forward(mq, orc):  # model.rs:882
    cfg = qwen3_tiny_config()
    recs = list(synth.random_model_records(cfg, 17, qk_norm=True))
    gm, om = both(mq, orc, cfg, recs)
    toks = [5, 11, 23, 97, 3, 42]
    ref = om.forward_full(toks)
    c = gm.new_cache()
    gm.forward(toks[:2], c)
    close(ref, gm.forward(toks[2:], c))


def test_qk_norm_actually_changes_output(mq):  # model.rs:903
    cfg = qwen3_tiny_config()
    recs = list(synth.random_model_records(cfg, 19, qk_norm=True))
    a = mq.Model.from_tensors(cfg, recs)
    b = mq.Model.from_tensors(cfg, [r for r in recs if "q_norm" not in r[0] and "k_norm" not in r[0]])
    d = np.abs(a.forward([1, 2, 3], a.new_cache()) - b.forward([1, 2, 3], b.new_cache())).max()
    assert d > 1e-3


def test_qkv_bias_path(mq, orc):
    cfg = ModelConfig(128, 256, 2, 4, 2, 32, 128, 64, 1e6, 1e-6, True, "q8_0")
    recs = quantize_records(synth.random_model_records(cfg, 9, with_bias=True), 1, orc)
    gm, om = both(mq, orc, cfg, recs)
    toks = [3, 1, 4, 1, 5, 9, 2, 6]
    close(om.forward_full(toks), gm.forward(toks, gm.new_cache()))


def test_forward_errors(mq, orc):  # model.rs:255-265, tensor.rs:73
    from minq_b200 import MinqError
    cfg = tiny_config(2)
    gm = mq.Model.from_tensors(cfg, synth.random_model_records(cfg, 5))
    c = gm.new_cache()
    with pytest.raises(MinqError, match="empty token sequence"):
        gm.forward([], c)
    with pytest.raises(MinqError, match="out of bounds"):
        gm.forward([128], c)
    gm.forward(list(range(64)), c)
    assert c.len == 64
    with pytest.raises(MinqError, match=r"exceeds max_seq_len \(64\)"):
        gm.forward([1], c)
    c.reset()
    assert c.len == 0
    gm.forward([1], c)


def test_missing_tensor_is_a_model_error(mq):
    from minq_b200 import MinqError
    cfg = tiny_config(2)
    recs = [r for r in synth.random_model_records(cfg, 5) if "k_proj" not in r[0]]
    with pytest.raises(MinqError, match="missing tensor"):
        mq.Model.from_tensors(cfg, recs)


@pytest.mark.parametrize("chunk", [None, 4096, 12304])
def test_load_minq_file(mq, orc, tmp_path, monkeypatch, chunk):  # model.rs:711 via format.rs
    """The mapped-file loader (pinned double buffers, one copy per chunk) with
    its default chunk and with chunks far smaller than the tensors, so every
    tensor crosses several buffers and both buffers recycle."""
    if chunk:
        monkeypatch.setenv("MINQ_LOAD_CHUNK_BYTES", str(chunk))
    cfg = tiny_config(2, dtype="q4_0", hidden=128, inter=256)
    recs = quantize_records(synth.random_model_records(cfg, 11), 2, orc)
    p = tmp_path / "tiny.minq"
    write_minq(p, cfg, recs)
    gm = mq.Model.load_minq(p)
    om = orc.Model.load_minq(str(p))
    toks = [9, 8, 7, 6]
    close(om.forward(toks, om.new_cache()), gm.forward(toks, gm.new_cache()))
    built = mq.Model.from_tensors(cfg, recs)
    assert np.array_equal(gm.forward(toks, gm.new_cache()), built.forward(toks, built.new_cache()))


def test_engine_generate_matches_oracle_greedy(mq, orc):  # engine.rs:98
    cfg = tiny_config(4, dtype="q8_0", hidden=128, inter=256)
    recs = quantize_records(synth.random_model_records(cfg, 1), 1, orc)
    gm, om = both(mq, orc, cfg, recs)
    seen = []
    stats = mq.Engine(gm, mq.Sampler.greedy()).generate([1, 2, 3], 16, seen.append)
    assert stats.gen_tokens == 16 and stats.prompt_tokens == 3
    ref, _ = orc.greedy_generate(om, [1, 2, 3], 16)
    assert seen == ref


def test_engine_rejects_empty_prompt_and_callback_errors(mq):  # engine.rs:119,126
    from minq_b200 import MinqError
    cfg = tiny_config(2)
    gm = mq.Model.from_tensors(cfg, synth.random_model_records(cfg, 6))
    eng = mq.Engine(gm, mq.Sampler.greedy())
    with pytest.raises(MinqError, match="empty prompt"):
        eng.generate([], 4)
    seen = []

    def cb(t):
        seen.append(t)
        if len(seen) == 2:
            raise RuntimeError("sink closed")

    with pytest.raises(RuntimeError, match="sink closed"):
        eng.generate([1, 2], 8, cb)
    assert len(seen) == 2


def test_engine_stop_tokens(mq):
    cfg = tiny_config(2)
    gm = mq.Model.from_tensors(cfg, synth.random_model_records(cfg, 6))
    eng = mq.Engine(gm, mq.Sampler.greedy())
    first = []
    eng.generate([1, 2], 1, first.append)
    eng.stop_tokens = [first[0]]
    seen = []
    st = eng.generate([1, 2], 8, seen.append)
    assert seen == first and st.gen_tokens == 1


def test_graph_replay_and_eager_launch_agree(mq, orc):
    """The captured-graph step (device-side position, capacity-sized attention
    grid) and the eager step give the same logits and cache."""
    cfg = tiny_config(2, dtype="q4_0", hidden=128, inter=256)
    recs = quantize_records(synth.random_model_records(cfg, 13), 2, orc)
    gm, om = both(mq, orc, cfg, recs)
    toks = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3]
    ca = gm.new_cache()
    a = gm.forward(toks, ca)
    gm.set_graphs(False)
    cb = gm.new_cache()
    b = gm.forward(toks, cb)
    gm.set_graphs(True)
    close(a, b, 1e-4)
    close(om.forward(toks, om.new_cache()), a)
    for layer in range(cfg.n_layers):
        assert np.abs(ca.read(layer)[0] - cb.read(layer)[0]).max() < 1e-5
    # mixing: eager steps then graph steps on one cache
    cc = gm.new_cache()
    gm.set_graphs(False)
    gm.forward(toks[:4], cc)
    gm.set_graphs(True)
    close(a, gm.forward(toks[4:], cc), 1e-4)


def test_decode_steps_matches_oracle_greedy(mq, orc):
    """minq_decode_steps (greedy continuation without the host in the loop)."""
    import torch
    cfg = tiny_config(4, dtype="q8_0", hidden=128, inter=256)
    recs = quantize_records(synth.random_model_records(cfg, 21), 1, orc)
    gm, om = both(mq, orc, cfg, recs)
    prompt = [7, 7, 3, 100, 42]
    ref, _ = orc.greedy_generate(om, prompt, 12)
    c = gm.new_cache()
    first = gm.forward_argmax(prompt, c)
    out = torch.zeros(11, dtype=torch.int32, device="cuda")
    gm.decode_steps(c, 11, out.data_ptr())
    torch.cuda.synchronize()
    got = [first] + [int(v) for v in out.cpu().numpy()]
    assert got == ref
    assert c.len == len(prompt) + 11


# ------------------------------------------------ benchmark architectures

def _greedy_parity(mq, orc, arch, prompt_len, n_tokens, max_seq, seed=1234):
    import torch
    cfg0, qk_norm, tied = synth.ARCH[arch]
    from dataclasses import replace
    cfg = replace(cfg0, max_seq_len=max_seq)
    recs = synth.to_host(synth.synth_records(cfg, seed, qk_norm, tied))
    torch.cuda.empty_cache()
    gm = mq.Model.from_tensors(cfg, recs)
    om = orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    del recs
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, prompt_len).astype(np.uint32)
    ref, margins = orc.greedy_generate(om, prompt, n_tokens)
    got = []
    mq.Engine(gm, mq.Sampler.greedy()).generate(prompt, n_tokens, got.append)
    if got != ref:
        i = next(j for j in range(n_tokens) if got[j] != ref[j])
        pytest.fail(f"{arch}: first greedy mismatch at step {i} (oracle top-2 margin "
                    f"{margins[i]:.3g}); gpu {got[:i + 1]} vs oracle {ref[:i + 1]}")


@pytest.mark.slow
def test_greedy_tokens_qwen2_0_5b_q8_0(mq, orc):
    """Benchmark config 1 shape: Qwen2-0.5B, Q8_0, prompt 128, 64 greedy tokens."""
    _greedy_parity(mq, orc, "qwen2-0.5b", 128, 64, 256)


@pytest.mark.slow
def test_greedy_tokens_qwen3_4b_q4_0(mq, orc):
    """Benchmark config 3 shape (Qwen3-4B, Q4_0, q/k-norm), short prompt, 64 tokens."""
    _greedy_parity(mq, orc, "qwen3-4b", 16, 64, 128)
