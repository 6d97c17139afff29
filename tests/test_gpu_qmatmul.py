"""The batched quantized product minq_qmatmul (QuantizedTensor::matvec,
quantize.rs:215-249, applied to every input of a batch) on the tensor cores
against the CPU oracle.

Tolerance (as for the single matvec): |gpu - ref| <= 1e-5 * sum_k |w_k x_k|
per row and input; ref is the oracle's matvec for a few inputs of each case
and the exact (float64) product of the dequantized weights for all of them
(the oracle itself sits within 1e-7 of that bound from the exact value).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = np.float32


def _case(orc, dt, rows, cols, B, seed, hdr=False):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(rows * cols).astype(F) * F(0.02)).astype(F)
    if hdr:
        # inputs spanning 2^-20 .. 1 inside every 32-column block, random signs
        e = rng.integers(-20, 1, size=(B, cols))
        x = (np.ldexp(1.0, e) * rng.choice([-1.0, 1.0], size=(B, cols))
             * (1 + rng.random((B, cols)))).astype(F)
    else:
        x = rng.standard_normal((B, cols)).astype(F)
    data = orc.quantize(dt, w)
    return data, x


def _check(mq, orc, dt, rows, cols, data, x):
    from minq_b200 import api
    B = x.shape[0]
    y = api.QuantizedTensor(dt, rows, cols, data).matmul(x)
    assert y.shape == (B, rows)
    assert mq._lib.lib().minq_device_status() == 0, "a bounded device wait timed out"
    wd = orc.dequantize(dt, data).reshape(rows, cols).astype(np.float64)
    exact = x.astype(np.float64) @ wd.T
    bound = np.abs(x.astype(np.float64)) @ np.abs(wd).T
    err = np.abs(y.astype(np.float64) - exact)
    assert np.all(err <= 1e-5 * bound + 1e-30), float((err / (bound + 1e-30)).max())
    for b in sorted({0, B - 1}):
        ref = orc.qmatvec(dt, data, rows, cols, x[b])
        e2 = np.abs(y[b].astype(np.float64) - ref)
        assert np.all(e2 <= 1e-5 * bound[b] + 1e-30), (b, float((e2 / (bound[b] + 1e-30)).max()))


CASES = [
    # dtype, rows, cols, batch
    (2, 256, 128, 2),        # one chunk, one row tile
    (2, 300, 896, 5),        # ragged row tile, 7 chunks
    (2, 17, 256, 16),        # fewer rows than a tile
    (2, 6144, 2560, 64),     # Qwen3-4B q|k|v at a 64-token prefill chunk
    (2, 2560, 9728, 33),     # Qwen3-4B down_proj
    (2, 4096, 4096, 64),     # LLaMA-3-8B q / o_proj, 64 sequences
    (2, 14336, 4096, 64),    # LLaMA-3-8B gate / up
    (2, 4096, 14336, 64),    # LLaMA-3-8B down_proj
    (2, 1024, 4096, 8),      # k / v at 8 sequences per GPU
    (1, 896, 896, 17),
    (1, 4864, 896, 32),
    (1, 2560, 4096, 64),
    (1, 129, 384, 3),
    # row tiles past one wave of SMs: 152 tiles = 148 + 4 (the 4 split over
    # the SMs in a second launch), and 224 tiles (every tile in K slices)
    (2, 19456, 512, 16),
    (2, 28672, 1024, 64),
]


@pytest.mark.parametrize("dt,rows,cols,B", CASES, ids=[f"{'q8' if c[0] == 1 else 'q4'}_{c[1]}x{c[2]}_b{c[3]}" for c in CASES])
def test_gpu_qmatmul_matches_oracle(mq, orc, dt, rows, cols, B):
    data, x = _case(orc, dt, rows, cols, B, rows * 31 + cols * 7 + B)
    _check(mq, orc, dt, rows, cols, data, x)


@pytest.mark.parametrize("dt", [1, 2])
def test_gpu_qmatmul_high_dynamic_range(mq, orc, dt):
    data, x = _case(orc, dt, 512, 1024, 24, 99 + dt, hdr=True)
    _check(mq, orc, dt, 512, 1024, data, x)


def test_gpu_qmatmul_single_input_and_zero_blocks(mq, orc):
    # one input (CUDA-core kernel) and all-zero weight blocks (d = 0)
    rows, cols = 64, 256
    w = np.zeros(rows * cols, F)
    w[: cols * 8] = np.random.default_rng(3).standard_normal(cols * 8).astype(F) * F(0.02)
    data = orc.quantize(2, w)
    for B in (1, 4):
        x = np.random.default_rng(B).standard_normal((B, cols)).astype(F)
        _check(mq, orc, 2, rows, cols, data, x)


def test_gpu_qmatmul_rejects(mq):
    from minq_b200 import api, MinqError
    qt = api.QuantizedTensor(2, 4, 64, np.zeros(4 * 2 * 20, np.uint8))
    with pytest.raises(MinqError, match=r"\[batch, 64\]"):
        qt.matmul(np.zeros((2, 63), F))
    with pytest.raises(MinqError, match="batch must be 1..64"):
        qt.matmul(np.zeros((65, 64), F))
