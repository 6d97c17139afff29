"""Generate tests/golden/golden.npz: fixed inputs and expected outputs for the
hot-path functions, from a restatement independent of the C++ oracle.

The reference (Rust) cannot be built here and ships no golden vectors, so
the expected values come from this second, numpy-based restatement:
  * quantize_q8_0 / quantize_q4_0 (quantize.rs:78-143) in numpy float32
    arithmetic (IEEE division / multiply, exact round-half-away-from-zero,
    clamp, NaN -> 0 saturating cast): bit-exact expected bytes;
  * RopeTables (model.rs:170-186) by calling glibc's powf / sinf / cosf
    through ctypes, the same libm the Rust reference calls: bit-exact;
  * matvec / attend / rmsnorm / softmax expectations in float64 from the
    dequantized weights (checked with a tolerance).
The inputs include the reference tests' own fixtures: the known-answer block
x_i = i - 16 (quantize.rs:444-457), the 4 x 64 matvec shape
(quantize.rs:460-475), the rmsnorm vector [1, 2, 3, 4] (tensor.rs:262-279)
and the softmax vector [1, 2, 3, 4, 100] (tensor.rs:282-289).

Run: python tests/golden/make_golden.py   (rewrites golden.npz)
"""
from __future__ import annotations

import ctypes
import ctypes.util
import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
F = np.float32

_libm = ctypes.CDLL(ctypes.util.find_library("m"))
for _n in ("powf", "sinf", "cosf"):
    getattr(_libm, _n).restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
_libm.sinf.argtypes = [ctypes.c_float]
_libm.cosf.argtypes = [ctypes.c_float]


def round_half_away(v: np.ndarray) -> np.ndarray:
    """Rust f32::round: exact, half away from zero (no x+0.5 rounding trap)."""
    with np.errstate(invalid="ignore"):
        t = np.trunc(v)
        frac = v - t
        bump = np.where(np.abs(frac) >= F(0.5), np.sign(v), F(0)).astype(F)
        return (t + bump).astype(F)


def _amax(b: np.ndarray) -> np.ndarray:
    # fold(0.0, f32::max) over |v|: NaN is skipped, start value 0.
    return np.fmax.reduce(np.abs(b), axis=1, initial=F(0)).astype(F)


def np_quantize(x: np.ndarray, q4: bool) -> np.ndarray:
    b = np.asarray(x, dtype=F).reshape(-1, 32)
    amax = _amax(b)
    d = (amax / F(8.0 if q4 else 127.0)).astype(F)
    out = []
    for i in range(b.shape[0]):
        dd = d[i]
        if q4:
            codes = np.zeros(32, dtype=np.int64)
            if dd != 0:
                with np.errstate(over="ignore", invalid="ignore"):
                    idv = F(1.0) / dd
                    r = round_half_away((b[i] * idv).astype(F))
                c = np.clip(r, -8, 7)
                c = np.where(np.isnan(c), 0, c).astype(np.int64)
                codes = c + 8
                packed = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)
            else:
                packed = np.zeros(16, dtype=np.uint8)
            out.append(np.frombuffer(np.float32(dd).tobytes(), dtype=np.uint8))
            out.append(packed)
        else:
            if dd != 0:
                with np.errstate(over="ignore", invalid="ignore"):
                    idv = F(1.0) / dd
                    r = round_half_away((b[i] * idv).astype(F))
                c = np.clip(r, -127, 127)
                c = np.where(np.isnan(c), 0, c).astype(np.int64)
                codes = c.astype(np.int8).view(np.uint8)
            else:
                codes = np.zeros(32, dtype=np.uint8)
            out.append(np.frombuffer(np.float32(dd).tobytes(), dtype=np.uint8))
            out.append(codes)
    return np.concatenate(out).astype(np.uint8)


def np_dequantize(data: np.ndarray, q4: bool) -> np.ndarray:
    bb = 20 if q4 else 36
    blk = data.reshape(-1, bb)
    d = blk[:, :4].copy().view(np.float32).reshape(-1)
    if q4:
        lo = (blk[:, 4:] & 0x0F).astype(np.int64) - 8
        hi = (blk[:, 4:] >> 4).astype(np.int64) - 8
        codes = np.empty((blk.shape[0], 32), dtype=np.int64)
        codes[:, 0::2], codes[:, 1::2] = lo, hi
    else:
        codes = blk[:, 4:].view(np.int8).astype(np.int64)
    return (codes.astype(F) * d[:, None]).astype(F).reshape(-1)


def rope_tables(hd: int, max_seq: int, theta: float):
    half = hd // 2
    cs = np.zeros((max_seq, half), dtype=F)
    sn = np.zeros((max_seq, half), dtype=F)
    for i in range(half):
        e = F(F(2.0) * F(i)) / F(hd)
        freq = F(1.0) / F(_libm.powf(F(theta), e))
        for pos in range(max_seq):
            ang = F(F(pos) * freq)
            sn[pos, i] = _libm.sinf(ang)
            cs[pos, i] = _libm.cosf(ang)
    return cs, sn


def attend64(q, k, v, n_heads, n_kv, hd):
    """model.rs:223-248 in float64."""
    q = q.astype(np.float64).reshape(n_heads, hd)
    L = k.shape[0]
    k = k.astype(np.float64).reshape(L, n_kv, hd)
    v = v.astype(np.float64).reshape(L, n_kv, hd)
    g = n_heads // n_kv
    out = np.zeros((n_heads, hd))
    for h in range(n_heads):
        s = k[:, h // g, :] @ q[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ v[:, h // g, :]
    return out.reshape(-1)


def main():
    rng = np.random.default_rng(20260101)
    g = {}
    # --- quantizer fixtures ---
    uni = ((rng.random(32 * 64, dtype=F) - F(0.5)) * F(2.0)).astype(F)
    known = (np.arange(32, dtype=F) - F(16)).astype(F)           # quantize.rs:446
    zeros = np.zeros(32, dtype=F)
    negz = np.full(32, -0.0, dtype=F)
    nan_one = uni[:32].copy(); nan_one[5] = np.nan
    all_nan = np.full(32, np.nan, dtype=F)
    tiny = np.full(32, F(1e-38), dtype=F); tiny[3] = F(-1e-38); tiny[7] = F(0)
    denorm = np.full(32, F(1e-44), dtype=F)
    ties8 = np.array([127, 2.5, -3.5, 0.5, -0.5, 1.5, -1.5, 126.5] + [0.25] * 24, dtype=F)
    ties4 = np.array([8, 2.5, -3.5, 0.5, -0.5, 1.5, -1.5, 6.5, -7.5, 7.5] + [0.25] * 22, dtype=F)
    big = (uni[:32] * F(1e30)).astype(F)
    inf_blk = uni[:32].copy(); inf_blk[0] = np.inf
    edge = np.concatenate([known, zeros, negz, nan_one, all_nan, tiny, denorm, ties8, ties4,
                           big, inf_blk]).astype(F)
    normal = (rng.standard_normal(32 * 64).astype(F) * F(0.02)).astype(F)
    for nm, x in [("uni", uni), ("edge", edge), ("normal", normal)]:
        g[f"q_in_{nm}"] = x
        g[f"q8_{nm}"] = np_quantize(x, False)
        g[f"q4_{nm}"] = np_quantize(x, True)
    # --- matvec fixtures (quantize.rs:460 shape 4x64 plus model-like shapes) ---
    for rows, cols in [(4, 64), (37, 96), (16, 896), (8, 2560)]:
        w = ((rng.random(rows * cols, dtype=F) - F(0.5)) * F(2.0)).astype(F)
        x = ((rng.random(cols, dtype=F) - F(0.5)) * F(2.0)).astype(F)
        tag = f"{rows}x{cols}"
        g[f"mv_x_{tag}"] = x
        g[f"mv_w_{tag}"] = w.reshape(rows, cols)
        for q4, qn in [(False, "q8"), (True, "q4")]:
            data = np_quantize(w, q4)
            g[f"mv_{qn}_w_{tag}"] = data
            wd = np_dequantize(data, q4).astype(np.float64).reshape(rows, cols)
            g[f"mv_{qn}_y_{tag}"] = wd @ x.astype(np.float64)
        g[f"mv_f32_y_{tag}"] = w.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
    # --- rmsnorm (tensor.rs:262) / softmax (tensor.rs:282) known answers ---
    g["rms_x"] = np.array([1, 2, 3, 4], dtype=F)
    g["rms_y"] = (np.array([1, 2, 3, 4], dtype=np.float64) / np.sqrt(30 / 4 + 1e-5))
    g["sm_x"] = np.array([1, 2, 3, 4, 100], dtype=F)
    e = np.exp(np.array([1, 2, 3, 4, 100], dtype=np.float64) - 100)
    g["sm_y"] = e / e.sum()
    # --- RoPE tables (model.rs:760 test params, and the 128-dim config) ---
    for hd, ms, th in [(16, 64, 10000.0), (128, 80, 1e6), (64, 40, 1e6)]:
        cs, sn = rope_tables(hd, ms, th)
        g[f"rope_cos_{hd}_{ms}"] = cs
        g[f"rope_sin_{hd}_{ms}"] = sn
    # --- attention (GQA) ---
    for nh, nkv, hd, L in [(4, 2, 16, 17), (14, 2, 64, 63), (32, 8, 128, 33), (4, 1, 8, 5)]:
        tag = f"{nh}_{nkv}_{hd}_{L}"
        q = rng.standard_normal(nh * hd).astype(F)
        k = rng.standard_normal((L, nkv * hd)).astype(F)
        v = rng.standard_normal((L, nkv * hd)).astype(F)
        g[f"att_q_{tag}"], g[f"att_k_{tag}"], g[f"att_v_{tag}"] = q, k, v
        g[f"att_o_{tag}"] = attend64(q, k, v, nh, nkv, hd)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
