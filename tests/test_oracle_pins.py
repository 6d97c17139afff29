"""Pins of the CPU oracle: the reference's own unit tests (quantize.rs,
tensor.rs, model.rs, sampler.rs, engine.rs), restated against the oracle,
plus the golden vectors of tests/golden (independent numpy/glibc
restatement). CPU only."""
import numpy as np
import pytest

from minq_b200.minq_format import ModelConfig
from minq_b200 import synth

F = np.float32


def rand_vec(n, seed):
    """quantize.rs:394 rand_vec: uniform [-1, 1)."""
    r = np.random.default_rng(seed)
    return ((r.random(n, dtype=F) - F(0.5)) * F(2.0)).astype(F)


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.sqrt(((a - b) ** 2).sum() / (a ** 2).sum())


# ---------------- quantize.rs tests ----------------

def test_q8_0_roundtrip_error_is_bounded(orc):  # quantize.rs:420
    x = rand_vec(32 * 64, 7)
    y = orc.dequantize(orc.Q8_0, orc.quantize_q8_0(x))
    assert rel_err(x, y) < 0.01


def test_q4_0_is_less_accurate_than_q8_0(orc):  # quantize.rs:430
    x = rand_vec(32 * 64, 11)
    r8 = rel_err(x, orc.dequantize(orc.Q8_0, orc.quantize_q8_0(x)))
    r4 = rel_err(x, orc.dequantize(orc.Q4_0, orc.quantize_q4_0(x)))
    assert r4 > r8
    assert r4 < 0.25


def test_q8_0_block_uses_full_scale(orc):  # quantize.rs:444 (known answer)
    x = (np.arange(32, dtype=F) - F(16)).astype(F)
    b = orc.quantize_q8_0(x)
    d = b[:4].view(np.float32)[0]
    assert abs(float(d) - 16.0 / 127.0) < 1e-9
    assert d == F(16.0) / F(127.0)
    y = orc.dequantize(orc.Q8_0, b)
    assert np.abs(x - y).max() <= d / 2 + 1e-6


def test_quantized_matvec_matches_dequantized_matvec(orc):  # quantize.rs:460
    w = rand_vec(4 * 64, 3).reshape(4, 64)
    x = rand_vec(64, 5)
    for dt in (orc.Q8_0, orc.Q4_0):
        data = orc.quantize(dt, w)
        fast = orc.qmatvec(dt, data, 4, 64, x)
        ref = orc.matvec_f32(orc.dequantize(dt, data).reshape(4, 64), x)
        assert np.abs(fast - ref).max() < 1e-3


def test_rejects_misaligned_input(orc):  # quantize.rs:478
    with pytest.raises(orc.OracleError):
        orc.quantize_q8_0(np.ones(17, F))
    with pytest.raises(orc.OracleError):
        orc.quantize_q4_0(np.ones(33, F))


@pytest.mark.parametrize("dt", [1, 2])
def test_avx2_row_matches_scalar(orc, dt):  # quantize.rs:486,501
    x = rand_vec(32 * 8, 21 if dt == 1 else 23)
    row = orc.quantize(dt, rand_vec(32 * 8, 22 if dt == 1 else 24))
    s = orc.qrow(dt, row, x, simd=False)
    v = orc.qrow(dt, row, x, simd=True)
    assert abs(s - v) / max(abs(s), 1e-6) < 1e-5


def test_quantizer_matches_golden(orc, golden):
    for nm in ("uni", "edge", "normal"):
        x = golden[f"q_in_{nm}"]
        assert np.array_equal(orc.quantize_q8_0(x), golden[f"q8_{nm}"]), nm
        assert np.array_equal(orc.quantize_q4_0(x), golden[f"q4_{nm}"]), nm


def test_q4_zero_block_packs_zero_bytes(orc):  # quantize.rs:127-139
    b = orc.quantize_q4_0(np.zeros(32, F))
    assert np.all(b == 0)


def test_matvec_matches_golden(orc, golden):
    for tag in ("4x64", "37x96", "16x896", "8x2560"):
        rows, cols = map(int, tag.split("x"))
        x = golden[f"mv_x_{tag}"]
        for qn, dt in (("q8", orc.Q8_0), ("q4", orc.Q4_0)):
            exp = golden[f"mv_{qn}_y_{tag}"]
            for simd in (True, False):
                orc.set_simd(simd)
                got = orc.qmatvec(dt, golden[f"mv_{qn}_w_{tag}"], rows, cols, x)
                scale = np.abs(exp).max() + 1e-6
                assert np.abs(got - exp).max() / scale < 1e-5, (tag, qn, simd)
        orc.set_simd(True)
        got = orc.matvec_f32(golden[f"mv_w_{tag}"], x)
        exp = golden[f"mv_f32_y_{tag}"]
        assert np.abs(got - exp).max() / (np.abs(exp).max() + 1e-6) < 1e-5


# ---------------- tensor.rs tests ----------------

def test_rmsnorm_matches_hand_computed_reference(orc, golden):  # tensor.rs:262
    x = golden["rms_x"]
    got = orc.rmsnorm(x, np.ones(4, F), 1e-5)
    assert np.abs(got - golden["rms_y"]).max() < 1e-6
    got2 = orc.rmsnorm(x, np.full(4, 2.0, F), 1e-5)
    assert np.abs(got2 - 2 * got).max() < 1e-6


def test_softmax_sums_to_one(orc, golden):  # tensor.rs:282
    v = orc.softmax(golden["sm_x"])
    assert abs(v.sum() - 1.0) < 1e-6
    assert v[4] > v[3] > v[2]
    assert np.abs(v - golden["sm_y"]).max() < 1e-6


@pytest.mark.parametrize("n", [1, 7, 8, 15, 16, 33, 64, 100, 1024])
def test_avx2_dot_matches_scalar(orc, n):  # tensor.rs:293
    i = np.arange(n, dtype=F)
    a = np.sin(i * F(0.37)).astype(F)
    b = np.cos(i * F(0.11)).astype(F)
    s, v = orc.dot(a, b, simd=False), orc.dot(a, b, simd=True)
    assert abs(s - v) / max(abs(s), 1e-6) < 1e-5


# ---------------- model.rs RoPE tests ----------------

def test_rope_preserves_vector_norm(orc):  # model.rs:748
    x = rand_vec(2 * 16, 1)
    y = orc.apply_rope(x, 37, 2, 16, 10000.0)
    assert abs(np.linalg.norm(x) - np.linalg.norm(y)) < 1e-4


def test_rope_tables_match_on_the_fly_computation(orc):  # model.rs:760 (bit-identical)
    cs, sn = orc.rope_tables(16, 64, 10000.0)
    for pos in (0, 1, 7, 33, 63):
        a = rand_vec(32, 100 + pos)
        assert np.array_equal(orc.apply_rope(a, pos, 2, 16, 10000.0),
                              orc.rope_apply_tables(cs, sn, a, pos))


def test_rope_tables_match_golden(orc, golden):
    for hd, ms, th in ((16, 64, 10000.0), (128, 80, 1e6), (64, 40, 1e6)):
        cs, sn = orc.rope_tables(hd, ms, th)
        assert np.array_equal(cs, golden[f"rope_cos_{hd}_{ms}"])
        assert np.array_equal(sn, golden[f"rope_sin_{hd}_{ms}"])


def test_rope_encodes_relative_positions(orc):  # model.rs:775
    q, k = rand_vec(16, 2), rand_vec(16, 3)
    m, n, d = 9, 3, 5
    d1 = orc.dot(orc.apply_rope(q, m, 1, 16, 1e4), orc.apply_rope(k, n, 1, 16, 1e4))
    d2 = orc.dot(orc.apply_rope(q, m + d, 1, 16, 1e4), orc.apply_rope(k, n + d, 1, 16, 1e4))
    assert abs(d1 - d2) < 1e-4


def test_attend_matches_golden(orc, golden):
    for tag in ("4_2_16_17", "14_2_64_63", "32_8_128_33", "4_1_8_5"):
        nh, nkv, hd, L = map(int, tag.split("_"))
        out = orc.attend(golden[f"att_q_{tag}"], golden[f"att_k_{tag}"], golden[f"att_v_{tag}"],
                         L, nh, nkv, hd)
        exp = golden[f"att_o_{tag}"]
        assert np.abs(out - exp).max() <= 1e-5 * np.linalg.norm(exp)


# ---------------- model.rs forward tests (tiny f32 models) ----------------

def tiny_config(n_kv):  # model.rs:723
    return ModelConfig(64, 128, 2, 4, n_kv, 16, 128, 64, 10000.0, 1e-5, False, "f32")


def qwen3_tiny_config():  # model.rs:850
    return ModelConfig(64, 128, 2, 4, 2, 8, 128, 64, 1e6, 1e-6, False, "f32")


def cfg_dict(c):
    return {k: getattr(c, k) for k in c.__dataclass_fields__}


def oracle_model(orc, cfg, seed, qk_norm=False, bias=False):
    recs = list(synth.random_model_records(cfg, seed, qk_norm=qk_norm, with_bias=bias))
    return orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs}), recs


def assert_logits_close(a, b, tol=1e-3):  # model.rs:932
    assert a.shape == b.shape
    assert np.abs(a - b).max() < tol


def test_kv_cache_matches_full_forward(orc):  # model.rs:798
    m, _ = oracle_model(orc, tiny_config(4), 7)
    toks = [5, 11, 23, 97, 3, 42]
    ref = m.forward_full(toks)
    c = m.new_cache()
    for t in toks:
        last = m.forward([t], c)
    assert_logits_close(ref, last)
    c = m.new_cache()
    m.forward(toks[:4], c)
    assert_logits_close(ref, m.forward(toks[4:], c))


def test_gqa_broadcast_matches_expanded_kv(orc):  # model.rs:819
    cfg = tiny_config(1)
    recs = list(synth.random_model_records(cfg, 42))
    gqa = orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    cfg4 = tiny_config(4)
    exp = {}
    for n, t, s, d in recs:
        if n.endswith(("k_proj.weight", "v_proj.weight")):
            d = np.concatenate([d] * 4, axis=0)
            s = [s[0] * 4, s[1]]
        exp[n] = (t, s, d)
    mha = orc.Model.from_tensors(cfg_dict(cfg4), exp)
    toks = [1, 2, 3, 4, 5]
    assert_logits_close(gqa.forward_full(toks), mha.forward_full(toks))


def test_qwen3_kv_cache_matches_full_forward(orc):  # model.rs:882
    m, _ = oracle_model(orc, qwen3_tiny_config(), 17, qk_norm=True)
    toks = [5, 11, 23, 97, 3, 42]
    ref = m.forward_full(toks)
    c = m.new_cache()
    for t in toks:
        last = m.forward([t], c)
    assert_logits_close(ref, last)
    c = m.new_cache()
    m.forward(toks[:2], c)
    assert_logits_close(ref, m.forward(toks[2:], c))


def test_qk_norm_actually_changes_output(orc):  # model.rs:903
    cfg = qwen3_tiny_config()
    recs = list(synth.random_model_records(cfg, 19, qk_norm=True))
    a = orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs})
    b = orc.Model.from_tensors(cfg_dict(cfg), {n: (t, s, d) for n, t, s, d in recs
                                               if "q_norm" not in n and "k_norm" not in n})
    diff = np.abs(a.forward_full([1, 2, 3]) - b.forward_full([1, 2, 3])).max()
    assert diff > 1e-3


def test_head_dim_decoupled_from_hidden_size(orc):  # model.rs:923
    m, _ = oracle_model(orc, qwen3_tiny_config(), 23, qk_norm=True)
    assert m.forward_full([7, 8, 9]).shape == (128,)


def test_forward_errors(orc):  # model.rs:255,260
    m, _ = oracle_model(orc, tiny_config(2), 5)
    c = m.new_cache()
    with pytest.raises(orc.OracleError):
        m.forward([], c)
    m.forward(list(range(64)), c)
    with pytest.raises(orc.OracleError, match="max_seq_len"):
        m.forward([1], c)


def test_greedy_generation_is_deterministic(orc):  # engine.rs:98
    m, _ = oracle_model(orc, tiny_config(4), 1)
    a, _ = orc.greedy_generate(m, [1, 2, 3], 16)
    b, _ = orc.greedy_generate(m, [1, 2, 3], 16)
    assert a == b and len(a) == 16


# ---------------- sampler.rs ----------------

def test_argmax_total_cmp_and_ties(orc):  # sampler.rs:10
    assert orc.argmax(np.array([1.0, 3.0, 3.0, 2.0], F)) == 1     # lowest index on ties
    assert orc.argmax(np.array([-0.0, 0.0], F)) == 1              # +0 > -0
    assert orc.argmax(np.array([1.0, np.nan, np.inf], F)) == 1     # +NaN sorts highest
    neg_nan = np.array([0xFFC00000], dtype=np.uint32).view(np.float32)[0]
    assert orc.argmax(np.array([neg_nan, -np.inf], F)) == 1        # -NaN sorts lowest
    assert orc.argmax(np.array([], F)) == 0


def test_attend_parallel_heads_bit_identical(orc):
    """The opt-in parallel-heads attend (used by the long-history checks) gives
    the same bits as the reference's serial loop over heads (model.rs:223-248)."""
    rng = np.random.default_rng(3)
    nh, nkv, hd, L = 32, 8, 128, 777
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal((L, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((L, nkv * hd)).astype(np.float32)
    serial = orc.attend(q, k, v, L, nh, nkv, hd)
    orc.set_attn_parallel(True)
    try:
        par = orc.attend(q, k, v, L, nh, nkv, hd)
    finally:
        orc.set_attn_parallel(False)
    assert np.array_equal(serial.view(np.uint32), par.view(np.uint32))
