"""GPU parity of the tensor-core prefill attention (minq_attend_prefill,
tcgen05 kind::tf32 with hi/lo split operands) against the oracle's attend,
called through the C ABI.

Token t of a chunk at position p0 + t attends over positions 0..=p0+t of a
head-major cache, as the reference's prompt loop calls attend once per token
(model.rs:259-268 -> model.rs:223-248). Tolerance: the f32 bar, max-abs <=
1e-4 * ||out|| per token (the split operands keep the products to about
2^-21 of |q||k|; the TF32 bar of 1e-2 is not needed).
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


def P(t):
    return C.c_void_p(t.data_ptr())


def _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq):
    from minq_b200 import _lib
    L = _lib.lib()
    qd = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    kd = torch.from_numpy(np.ascontiguousarray(kc)).cuda()
    vd = torch.from_numpy(np.ascontiguousarray(vc)).cuda()
    out = torch.full((T, nh, hd), float("nan"), dtype=torch.float32, device="cuda")
    wsb = L.minq_attn_prefill_workspace_bytes(T, nh, nkv, hd)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
    _lib.check(L.minq_attend_prefill(P(qd), P(kd), P(vd), max_seq * hd, p0, T, nh, nkv, hd,
                                     P(out), P(ws), wsb, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _case(seed, p0, T, nh, nkv, hd, extra=0):
    rng = np.random.default_rng(seed)
    max_seq = p0 + T + extra
    kc = rng.standard_normal((nkv, max_seq, hd)).astype(F)
    vc = rng.standard_normal((nkv, max_seq, hd)).astype(F)
    q = rng.standard_normal((T, nh, hd)).astype(F)
    return q, kc, vc, max_seq


def _check_tokens(orc, got, q, kc, vc, p0, T, nh, nkv, hd, tokens=None):
    for t in (range(T) if tokens is None else tokens):
        n = p0 + t + 1
        kf = np.ascontiguousarray(kc[:, :n, :].transpose(1, 0, 2).reshape(n, nkv * hd))
        vf = np.ascontiguousarray(vc[:, :n, :].transpose(1, 0, 2).reshape(n, nkv * hd))
        ref = orc.attend(q[t].reshape(-1), kf, vf, n, nh, nkv, hd)
        err = np.abs(got[t].reshape(-1) - ref).max()
        assert err <= 1e-4 * np.linalg.norm(ref), (t, err, np.linalg.norm(ref))


@pytest.mark.parametrize("nh,nkv,hd,p0,T", [
    (32, 8, 128, 0, 64),      # first chunk of a prompt: one key tile, causal inside it
    (32, 8, 128, 5, 17),      # ragged: neither p0 nor T on a tile boundary
    (32, 8, 128, 1984, 64),   # the last chunk of a 2048-token prompt (split keys)
    (32, 8, 128, 4031, 64),   # many key tiles per split
    (14, 2, 64, 100, 64),     # Qwen2-0.5B shape: 7 query heads per kv head
    (8, 8, 64, 0, 1),         # one token, no GQA
    (16, 2, 128, 300, 33),
    (4, 1, 128, 70, 64),      # one kv head: a single M tile of 128 rows + splits
    (64, 8, 64, 63, 64),      # G = 8: four M tiles per kv head
])
def test_prefill_attention_matches_oracle(mq, orc, torch, nh, nkv, hd, p0, T):
    q, kc, vc, max_seq = _case(nh * 7 + p0 + T + hd, p0, T, nh, nkv, hd, extra=3)
    got = _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq)
    assert np.isfinite(got).all()
    # long histories: every fourth token plus the first and last (oracle time)
    toks = None if p0 + T < 1024 else sorted(set(range(0, T, 4)) | {T - 1})
    _check_tokens(orc, got, q, kc, vc, p0, T, nh, nkv, hd, toks)


def test_prefill_attention_large_scores(mq, orc, torch):
    """Scores of magnitude ~100 (peaked softmax): the running max moves across
    tiles and the O rescale in tensor memory carries the result."""
    nh, nkv, hd, p0, T = 32, 8, 128, 700, 64
    q, kc, vc, max_seq = _case(99, p0, T, nh, nkv, hd)
    q *= 8.0
    kc[:, ::97, :] *= 3.0  # a few dominant keys spread over the history
    got = _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq)
    _check_tokens(orc, got, q, kc, vc, p0, T, nh, nkv, hd, range(0, T, 3))


def test_prefill_attention_repeatable(mq, torch):
    """Two calls on the same inputs give identical bits (no order depends on
    timing: fixed splits, serial per-row softmax, fixed combine order)."""
    nh, nkv, hd, p0, T = 32, 8, 128, 1000, 64
    q, kc, vc, max_seq = _case(5, p0, T, nh, nkv, hd)
    a = _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq)
    b = _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_prefill_attention_equals_per_token_decode_kernel(mq, torch):
    """The tensor-core kernel against the library's own split-KV attention
    (minq_attend, one token at a time): same arithmetic contract, so both sit
    within the f32 bar of each other."""
    from minq_b200 import _lib
    L = _lib.lib()
    nh, nkv, hd, p0, T = 32, 8, 128, 250, 40
    q, kc, vc, max_seq = _case(11, p0, T, nh, nkv, hd)
    got = _prefill_gpu(torch, q, kc, vc, p0, T, nh, nkv, hd, max_seq)
    for t in (0, 13, T - 1):
        n = p0 + t + 1
        kf = torch.from_numpy(np.ascontiguousarray(
            kc[:, :n, :].transpose(1, 0, 2).reshape(n, nkv * hd))).cuda()
        vf = torch.from_numpy(np.ascontiguousarray(
            vc[:, :n, :].transpose(1, 0, 2).reshape(n, nkv * hd))).cuda()
        qd = torch.from_numpy(np.ascontiguousarray(q[t].reshape(-1))).cuda()
        out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
        wsb = L.minq_attn_workspace_bytes(1, nh, n)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        _lib.check(L.minq_attend(P(qd), P(kf), P(vf), n, nh, nkv, hd, P(out), P(ws), wsb, None))
        ref = out.cpu().numpy()
        assert np.abs(got[t].reshape(-1) - ref).max() <= 1e-4 * np.linalg.norm(ref)
