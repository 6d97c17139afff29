"""GPU parity of the hot-path kernels against the CPU oracle and the golden
vectors, called through the C ABI (libminq_cuda.so).

Tolerances:
  * quantize / dequantize / argmax / RoPE tables: bit-exact;
  * matvec: |gpu - oracle| <= 1e-5 * sum_j |w_ij x_j| per row (f32
    accumulation-order difference only);
  * attention: max-abs <= 1e-4 * ||out|| (f32 bar of the acceptance criteria).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = np.float32


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    return _t


def dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def P(t):
    return C.c_void_p(t.data_ptr())


# ---------------------------------------------------------------- quantize

def test_gpu_quantize_bit_exact_golden(mq, golden):
    from minq_b200 import api
    for nm in ("uni", "edge", "normal"):
        x = golden[f"q_in_{nm}"]
        assert np.array_equal(api.quantize_q8_0(x), golden[f"q8_{nm}"]), nm
        assert np.array_equal(api.quantize_q4_0(x), golden[f"q4_{nm}"]), nm


@pytest.mark.parametrize("n,scale", [(32, 1.0), (32 * 1000, 0.02), (32 * 100_003, 3.0),
                                     (32 * 4096, 1e-30)])
def test_gpu_quantize_matches_oracle(mq, orc, n, scale):
    from minq_b200 import api
    x = (np.random.default_rng(n).standard_normal(n).astype(F) * F(scale)).astype(F)
    x[::97] = 0.0
    assert np.array_equal(api.quantize_q8_0(x), orc.quantize_q8_0(x))
    assert np.array_equal(api.quantize_q4_0(x), orc.quantize_q4_0(x))


def test_gpu_dequantize_bit_exact(mq, orc, golden):
    from minq_b200 import api
    for nm in ("uni", "normal"):
        b8, b4 = golden[f"q8_{nm}"], golden[f"q4_{nm}"]
        assert np.array_equal(api.dequantize_q8_0(b8).view(np.uint32),
                              orc.dequantize(orc.Q8_0, b8).view(np.uint32))
        assert np.array_equal(api.dequantize_q4_0(b4).view(np.uint32),
                              orc.dequantize(orc.Q4_0, b4).view(np.uint32))


def test_gpu_quantize_rejects_misaligned(mq):
    from minq_b200 import api, MinqError
    with pytest.raises(MinqError, match="multiple of 32"):
        api.quantize_q8_0(np.ones(17, F))


# ---------------------------------------------------------------- matvec

def _bound(dt, data, rows, cols, x, orc):
    w = orc.dequantize(dt, data).reshape(rows, cols).astype(np.float64)
    return np.abs(w) @ np.abs(x.astype(np.float64))


def test_gpu_qmatvec_golden(mq, orc, golden):
    from minq_b200 import api
    for tag in ("4x64", "37x96", "16x896", "8x2560"):
        rows, cols = map(int, tag.split("x"))
        x = golden[f"mv_x_{tag}"]
        for qn, dt in (("q8", 1), ("q4", 2)):
            data = golden[f"mv_{qn}_w_{tag}"]
            y = api.QuantizedTensor(dt, rows, cols, data).matvec(x)
            exp = golden[f"mv_{qn}_y_{tag}"]
            assert np.all(np.abs(y - exp) <= 1e-5 * _bound(dt, data, rows, cols, x, orc) + 1e-30)


SHAPES = [(1, 32), (3, 64), (17, 96), (5, 160), (63, 224), (896, 896), (128, 896), (4864, 896),
          (896, 4864), (6144, 2560), (2560, 4096), (2560, 9728), (1024, 4096), (4096, 14336)]


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("dt", [1, 2])
def test_gpu_qmatvec_matches_oracle(mq, orc, rows, cols, dt):
    from minq_b200 import api
    rng = np.random.default_rng(rows * 7 + cols)
    w = (rng.standard_normal(rows * cols).astype(F) * F(0.02)).astype(F)
    x = rng.standard_normal(cols).astype(F)
    data = orc.quantize(dt, w)
    y = api.QuantizedTensor(dt, rows, cols, data).matvec(x)
    ref = orc.qmatvec(dt, data, rows, cols, x)
    bound = _bound(dt, data, rows, cols, x, orc)
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * bound + 1e-30), float((err / (bound + 1e-30)).max())


def test_gpu_qmatvec_rejects_shape(mq):
    from minq_b200 import api, MinqError
    qt = api.QuantizedTensor(1, 4, 64, np.zeros(4 * 2 * 36, np.uint8))
    with pytest.raises(MinqError, match="64 cols vs input len 63"):
        qt.matvec(np.zeros(63, F))


@pytest.mark.parametrize("rows,cols", [(4, 64), (37, 96), (1000, 896), (151936, 896), (3, 2560)])
def test_gpu_f32_matvec_matches_oracle(mq, orc, rows, cols):
    from minq_b200 import api
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)).astype(F) * F(0.02)).astype(F)
    x = rng.standard_normal(cols).astype(F)
    y = api.matvec_f32(w, x)
    ref = orc.matvec_f32(w, x)
    bound = np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64))
    assert np.all(np.abs(y - ref) <= 1e-5 * bound + 1e-30)


def test_gpu_argmax_total_cmp(mq, orc):
    from minq_b200 import api
    neg_nan = np.array([0xFFC00000], dtype=np.uint32).view(F)[0]
    cases = [np.array([1.0, 3.0, 3.0, 2.0], F), np.array([-0.0, 0.0], F),
             np.array([1.0, np.nan, np.inf], F), np.array([neg_nan, -np.inf], F),
             np.full(151936, 0.5, F)]
    big = np.random.default_rng(0).standard_normal(151936).astype(F)
    big[77777] = big.max()
    big[123] = big.max()
    cases.append(big)
    for c in cases:
        assert api.argmax(c) == orc.argmax(c)


# ---------------------------------------------------------------- attention

def _attend_gpu(torch, mq, q, k, v, L, nh, nkv, hd):
    from minq_b200 import _lib
    qd, kd, vd = dev(torch, q), dev(torch, k), dev(torch, v)
    out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    wsb = _lib.lib().minq_attn_workspace_bytes(1, nh, L)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().minq_attend(P(qd), P(kd), P(vd), L, nh, nkv, hd, P(out), P(ws), wsb,
                                      None))
    return out.cpu().numpy()


def test_gpu_attend_golden(mq, golden, torch):
    for tag in ("4_2_16_17", "14_2_64_63", "32_8_128_33", "4_1_8_5"):
        nh, nkv, hd, L = map(int, tag.split("_"))
        out = _attend_gpu(torch, mq, golden[f"att_q_{tag}"], golden[f"att_k_{tag}"],
                          golden[f"att_v_{tag}"], L, nh, nkv, hd)
        exp = golden[f"att_o_{tag}"]
        assert np.abs(out - exp).max() <= 1e-4 * np.linalg.norm(exp), tag


@pytest.mark.parametrize("nh,nkv,hd,L", [(4, 4, 16, 1), (4, 2, 16, 2), (14, 2, 64, 31),
                                         (14, 2, 64, 700), (32, 8, 128, 1), (32, 8, 128, 33),
                                         (32, 8, 128, 2049), (32, 8, 128, 8192), (32, 8, 128, 32768),
                                         (4, 1, 8, 70),
                                         (16, 1, 32, 300), (64, 4, 256, 129)])
def test_gpu_attend_matches_oracle(mq, orc, torch, nh, nkv, hd, L):
    rng = np.random.default_rng(nh * L + hd)
    q = rng.standard_normal(nh * hd).astype(F)
    k = rng.standard_normal((L, nkv * hd)).astype(F)
    v = rng.standard_normal((L, nkv * hd)).astype(F)
    out = _attend_gpu(torch, mq, q, k, v, L, nh, nkv, hd)
    ref = orc.attend(q, k, v, L, nh, nkv, hd)
    assert np.abs(out - ref).max() <= 1e-4 * np.linalg.norm(ref)


@pytest.mark.parametrize("B,L,qk_norm", [(1, 512, False), (8, 512, True), (1, 2048, True),
                                         (64, 512, False), (8, 8192, False), (64, 2048, True),
                                         (1, 32768, False)])
def test_gpu_attn_decode_step_matches_oracle(mq, orc, torch, B, L, qk_norm):
    """Decode-attention op (GQA 32/8, hd 128): RoPE(theta 1e6) on q and the new k at
    pos = L, optional q/k RMSNorm, append, attend over L+1 positions — against the
    oracle's per_head_norm + RopeTables + attend for every sequence. From B = 8 /
    L = 8192 and B = 64 / L = 512 on, the balanced (stream-K) plan runs."""
    _attn_decode_check(orc, torch, B, L, qk_norm, 32, 8, 128, range(B))


@pytest.mark.parametrize("nh,nkv,hd,B,L", [(14, 2, 64, 64, 6000), (32, 2, 128, 16, 3000),
                                           (8, 8, 256, 16, 4000)])
def test_gpu_attn_balanced_plan_head_layouts(mq, orc, torch, nh, nkv, hd, B, L):
    """The balanced (stream-K) plan on other head layouts: head_dim 64 (32-position
    tiles), 16 query heads per kv head (two query groups of 8), head_dim 256 with
    one query head per kv head; ragged last tiles. Sequences at both ends and one
    in the middle are checked against the oracle."""
    orc.set_attn_parallel(True)
    try:
        _attn_decode_check(orc, torch, B, L, False, nh, nkv, hd, (0, B // 2 + 1, B - 1))
    finally:
        orc.set_attn_parallel(False)


def _attn_decode_check(orc, torch, B, L, qk_norm, nh, nkv, hd, check):
    from minq_b200 import _lib
    eps = 1e-6
    rng = np.random.default_rng(B * 1000 + L)
    max_seq = L + 1
    cs, sn = orc.rope_tables(hd, max_seq, 1e6)
    kc = rng.standard_normal((B, nkv, max_seq, hd)).astype(F)
    vc = rng.standard_normal((B, nkv, max_seq, hd)).astype(F)
    q = rng.standard_normal((B, nh, hd)).astype(F)
    kn = rng.standard_normal((B, nkv, hd)).astype(F)
    vn = rng.standard_normal((B, nkv, hd)).astype(F)
    qg = (0.5 + rng.random(hd)).astype(F) if qk_norm else None
    kg = (0.5 + rng.random(hd)).astype(F) if qk_norm else None
    d = {n: dev(torch, a) for n, a in dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, cs=cs, sn=sn).items()}
    if qk_norm:
        d["qg"], d["kg"] = dev(torch, qg), dev(torch, kg)
    out = torch.empty((B, nh, hd), dtype=torch.float32, device="cuda")
    wsb = _lib.lib().minq_attn_workspace_bytes(B, nh, L + 1)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().minq_attn_decode(
        P(d["q"]), P(d["kn"]), P(d["vn"]), P(d["qg"]) if qk_norm else None,
        P(d["kg"]) if qk_norm else None, eps, P(d["cs"]), P(d["sn"]), B, nh, nkv, hd, L,
        P(d["kc"]), P(d["vc"]), nkv * max_seq * hd, max_seq * hd, hd, P(out), P(ws), wsb, None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    kc_after = d["kc"].cpu().numpy()
    for b in check:
        qb, kb = q[b].reshape(-1).copy(), kn[b].reshape(-1).copy()
        if qk_norm:
            qb = orc.per_head_norm(qb, qg, eps, hd)
            kb = orc.per_head_norm(kb, kg, eps, hd)
        qb = orc.rope_apply_tables(cs, sn, qb, L)
        kb = orc.rope_apply_tables(cs, sn, kb, L)
        # the appended key must equal the oracle's rotated key (per-element ops)
        assert np.abs(kc_after[b, :, L, :].reshape(-1) - kb).max() <= 1e-5 * np.abs(kb).max()
        hist_k = kc[b].transpose(1, 0, 2).reshape(max_seq, nkv * hd).copy()
        hist_v = vc[b].transpose(1, 0, 2).reshape(max_seq, nkv * hd).copy()
        hist_k[L] = kb
        hist_v[L] = vn[b].reshape(-1)
        ref = orc.attend(qb, hist_k, hist_v, L + 1, nh, nkv, hd)
        assert np.abs(got[b].reshape(-1) - ref).max() <= 1e-4 * np.linalg.norm(ref), b
