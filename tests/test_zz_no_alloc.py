"""minq_attend_static (the allocation-free attention entry point) against
minq_attend with a caller workspace and against the oracle, through the C ABI.

The file name sorts last so the entry point also runs after every other GPU
test of the session (the scratch's set-up then happens on a device that other
entry points have already used); it passes when run alone as well.
"""
import ctypes as C

import numpy as np
import pytest

F = np.float32
P = C.c_void_p


def _ptr(t):
    return P(t.data_ptr())


def _inputs(seed, L, nh, nkv, hd):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(nh * hd).astype(F)
    k = rng.standard_normal((L, nkv * hd)).astype(F)
    v = rng.standard_normal((L, nkv * hd)).astype(F)
    return q, k, v


def _attend_ws(torch, lib, qd, kd, vd, L, nh, nkv, hd):
    from minq_b200 import _lib
    out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    wsb = lib.minq_attn_workspace_bytes(1, nh, L)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    _lib.check(lib.minq_attend(_ptr(qd), _ptr(kd), _ptr(vd), L, nh, nkv, hd, _ptr(out),
                               _ptr(ws), wsb, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("nh,nkv,hd,L", [(32, 8, 128, 1), (32, 8, 128, 2049), (14, 2, 64, 700),
                                         (4, 1, 16, 300), (32, 8, 128, 32768)])
def test_gpu_attend_static_matches_workspace_entry(mq, orc, nh, nkv, hd, L):
    import torch
    from minq_b200 import _lib
    lib = _lib.lib()
    q, k, v = _inputs(nh * 7 + L, L, nh, nkv, hd)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    want = _attend_ws(torch, lib, qd, kd, vd, L, nh, nkv, hd)
    outs = []
    for _ in range(2):  # two calls in a row reuse the same static scratch
        out = torch.full((nh * hd,), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(lib.minq_attend_static(_ptr(qd), _ptr(kd), _ptr(vd), L, nh, nkv, hd,
                                          _ptr(out), None))
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    tol = 1e-6 * np.linalg.norm(want)
    for got in outs:
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() <= tol
    if L <= 2049:
        ref = orc.attend(q, k, v, L, nh, nkv, hd)
        assert np.abs(outs[1] - ref).max() <= 1e-4 * np.linalg.norm(ref)


@pytest.mark.gpu
def test_gpu_attend_static_back_to_back_different_shapes(mq, orc):
    """Two calls queued on one stream without a sync in between, with different
    lengths and head layouts: the second must not see the first's partials."""
    import torch
    from minq_b200 import _lib
    lib = _lib.lib()
    cases = [(32, 8, 128, 4000), (14, 2, 64, 333)]
    outs, refs = [], []
    for nh, nkv, hd, L in cases:
        q, k, v = _inputs(L, L, nh, nkv, hd)
        qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
        _lib.check(lib.minq_attend_static(_ptr(qd), _ptr(kd), _ptr(vd), L, nh, nkv, hd,
                                          _ptr(out), None))
        outs.append((out, qd, kd, vd))
        refs.append(orc.attend(q, k, v, L, nh, nkv, hd))
    torch.cuda.synchronize()
    for (out, *_), ref in zip(outs, refs):
        got = out.cpu().numpy()
        assert np.abs(got - ref).max() <= 1e-4 * np.linalg.norm(ref)


def test_attend_static_rejects_oversize_before_any_launch(mq):
    """Sizes beyond the static scratch are refused with a clear error, before
    the device is touched (runs without a GPU)."""
    from minq_b200 import _lib
    lib = _lib.lib()
    dummy = P(256)  # never dereferenced: the size check comes first
    st = lib.minq_attend_static(dummy, dummy, dummy, 1 << 20, 32, 8, 128, dummy, None)
    assert st == _lib.ERR_ARG
    msg = lib.minq_last_error().decode()
    assert "static scratch" in msg and "minq_attend" in msg


def test_attend_static_rejects_unsupported_heads_as_shape(mq):
    """head_dim > 256 and n_heads > 4096 are shape errors with minq_attend's
    wording even when their scratch would fit (runs without a GPU)."""
    from minq_b200 import _lib
    lib = _lib.lib()
    dummy = P(256)
    st = lib.minq_attend_static(dummy, dummy, dummy, 4, 2, 1, 512, dummy, None)
    assert st == _lib.ERR_SHAPE
    assert "unsupported head_dim 512" in lib.minq_last_error().decode()
    st = lib.minq_attend_static(dummy, dummy, dummy, 4, 8192, 8192, 8, dummy, None)
    assert st == _lib.ERR_SHAPE
    assert "n_heads" in lib.minq_last_error().decode()


@pytest.mark.gpu
def test_gpu_attend_static_status_word_reads_clear(mq):
    """After completed calls the entry point's own timeout word reads clear,
    through its getter and through minq_device_status."""
    import torch
    from minq_b200 import _lib
    lib = _lib.lib()
    q, k, v = _inputs(5, 900, 8, 2, 64)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty(8 * 64, dtype=torch.float32, device="cuda")
    for _ in range(3):
        _lib.check(lib.minq_attend_static(_ptr(qd), _ptr(kd), _ptr(vd), 900, 8, 2, 64,
                                          _ptr(out), None))
    assert lib.minq_attend_static_status() == _lib.OK
    assert lib.minq_device_status() == _lib.OK
