"""The oracle's Sampler (sampler.rs:20-109) and its StdRng, on the CPU.

Pins: the ChaCha block function against the ChaCha20 keystream test vectors
for the all-zero key and nonce, blocks 0 and 1 (RFC 7539 appendix A.1, test
vectors 1 and 2); the reference's own sampler tests (sampler.rs:121-160:
top_k = 1 and temperature 0 equal the argmax, equal seeds give equal
sequences, draws stay inside the vocabulary, top-p keeps the dominant token);
and two independent Python restatements checked against the oracle: the RNG
stream (PCG32 seed expansion, ChaCha12 four-block refills, rand's f32
conversion) and the sampling steps in f32 on the oracle's own softmax.

The PCG32 expansion, the ChaCha word layout and the f32 conversion follow
rand_core 0.6.4 / rand_chacha 0.3.1 / rand 0.8.8 as published; no output of
the reference itself pins them (parity of the RNG with rand is unpinned
beyond the block function)."""
import numpy as np
import pytest

M32, M64 = 0xFFFFFFFF, (1 << 64) - 1

# ChaCha20, all-zero key and nonce: keystream blocks 0 and 1 (RFC 7539 A.1)
CHACHA20_ZERO = [
    "76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
    "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586",
    "9f07e7be5551387a98ba977c732d080dcb0f29a048e3656912c6533e32ee7aed"
    "29b721769ce64e43d57133b074d839d531ed1f28510afb45ace10a1f4b794d6f",
]


def test_chacha_block_matches_chacha20_test_vectors(orc):
    for ctr, hexs in enumerate(CHACHA20_ZERO):
        out = orc.chacha_block(np.zeros(8, np.uint32), ctr, 0, 20)
        assert out.astype("<u4").tobytes().hex() == hexs


def _rotl(x, r):
    return ((x << r) | (x >> (32 - r))) & M32


def _py_block(key, ctr, rounds):
    s = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + list(key) + [
        ctr & M32, ctr >> 32, 0, 0]
    x = list(s)

    def qr(a, b, c, d):
        x[a] = (x[a] + x[b]) & M32; x[d] = _rotl(x[d] ^ x[a], 16)
        x[c] = (x[c] + x[d]) & M32; x[b] = _rotl(x[b] ^ x[c], 12)
        x[a] = (x[a] + x[b]) & M32; x[d] = _rotl(x[d] ^ x[a], 8)
        x[c] = (x[c] + x[d]) & M32; x[b] = _rotl(x[b] ^ x[c], 7)

    for _ in range(rounds // 2):
        qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15)
        qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14)
    return [(a + b) & M32 for a, b in zip(x, s)]


def py_stdrng_u32(seed, n):
    """rand 0.8 StdRng::seed_from_u64(seed), n x next_u32 (pure Python)."""
    st, key = seed, []
    for _ in range(8):
        st = (st * 6364136223846793005 + 11634580027462260723) & M64
        xs = (((st >> 18) ^ st) >> 27) & M32
        rot = st >> 59
        key.append(((xs >> rot) | (xs << ((32 - rot) & 31))) & M32)
    out, block = [], 0
    while len(out) < n:
        for b in range(4):
            out += _py_block(key, block + b, 12)
        block += 4
    return np.array(out[:n], dtype=np.uint32)


@pytest.mark.parametrize("seed", [0, 42, 123, 2**63 + 5])
def test_rng_stream_matches_python_restatement(orc, seed):
    s = orc.Sampler(1.0, 0, 1.0, seed)
    got = np.concatenate([s.rng_u32(70), s.rng_u32(130)])  # across refills
    assert np.array_equal(got, py_stdrng_u32(seed, 200))


def _logits(n, seed, scale=20.0):
    return ((np.random.default_rng(seed).random(n, dtype=np.float32) - 0.5) * scale).astype(
        np.float32)


def test_top_k_1_equals_greedy(orc):  # sampler.rs:121-126
    x = _logits(128, 1)
    assert orc.Sampler(1.0, 1, 1.0, 123).sample(x) == orc.argmax(x)


def test_temperature_zero_equals_greedy(orc):  # sampler.rs:128-133
    x = _logits(128, 2)
    assert orc.Sampler(0.0, 0, 1.0, 123).sample(x) == orc.argmax(x)


def test_sampling_is_reproducible_for_same_seed(orc):  # sampler.rs:135-143
    x = _logits(256, 3)
    a, b = orc.Sampler(0.8, 40, 0.9, 42), orc.Sampler(0.8, 40, 0.9, 42)
    assert [a.sample(x) for _ in range(32)] == [b.sample(x) for _ in range(32)]


def test_samples_are_within_vocabulary(orc):  # sampler.rs:145-151
    x = _logits(50, 4)
    s = orc.Sampler(1.0, 0, 1.0, 7)
    assert all(0 <= s.sample(x) < 50 for _ in range(64))


def test_top_p_keeps_at_least_one_candidate(orc):  # sampler.rs:153-160
    x = np.full(32, -100.0, dtype=np.float32)
    x[5] = 100.0
    assert orc.Sampler(1.0, 0, 0.5, 9).sample(x) == 5


def py_sample(orc, logits, t, top_k, top_p, u):
    """sampler.rs:47-109 in f32 with the oracle's softmax; u = the uniform."""
    f = np.float32
    n = len(logits)
    if t <= 0 or top_k == 1:
        return orc.argmax(logits)
    probs = orc.softmax((logits / f(t)).astype(np.float32))
    if (top_k == 0 or top_k >= n) and top_p >= 1.0:
        r = f(u)
        for i in range(n):
            r = f(r - probs[i])
            if r <= 0:
                return i
        return n - 1
    k = n if top_k == 0 else min(top_k, n)
    ranked = sorted(range(n), key=lambda i: (-float(probs[i]), i))[:k]
    cutoff, cum = k, f(0)
    for r, i in enumerate(ranked):
        cum = f(cum + probs[i])
        if cum >= f(top_p):
            cutoff = r + 1
            break
    total = f(0)
    for i in ranked[:cutoff]:
        total = f(total + probs[i])
    r = f(f(u) * total)
    for i in ranked[:cutoff]:
        r = f(r - probs[i])
        if r <= 0:
            return i
    return ranked[cutoff - 1]


@pytest.mark.parametrize("t,top_k,top_p", [(1.0, 0, 1.0), (0.8, 40, 0.9), (1.3, 0, 0.5),
                                           (0.7, 5, 1.0), (1.0, 300, 0.95)])
def test_oracle_sampler_matches_python_restatement(orc, t, top_k, top_p):
    x = _logits(300, 11, 8.0)
    x[17] = x[18]  # a tie
    s = orc.Sampler(t, top_k, top_p, 77)
    us = (py_stdrng_u32(77, 64) >> 8).astype(np.float64) * 2.0 ** -24
    for d in range(64):
        assert s.sample(x) == py_sample(orc, x, t, top_k, top_p, np.float32(us[d])), d


def _exact_draws(x, t, top_p, us):
    """The sampling steps in exact (f64) cumulative arithmetic on f32
    probabilities: the first position (index order without filters, rank
    order with top_p) whose cumulative mass reaches u (u * the kept mass)."""
    xt = x / np.float32(t)
    e = np.exp((xt - xt.max()).astype(np.float64))
    prob = (e / e.sum()).astype(np.float32).astype(np.float64)
    if top_p >= 1.0:
        cum = np.cumsum(prob)
        return [int(min(np.searchsorted(cum, u), len(x) - 1)) for u in us], np.arange(len(x))
    order = np.lexsort((np.arange(len(x)), -prob))
    cum = np.cumsum(prob[order])
    cutoff = int(np.searchsorted(cum, top_p)) + 1
    toks = [int(order[min(np.searchsorted(cum[:cutoff], u * cum[cutoff - 1]), cutoff - 1)])
            for u in us]
    pos = np.empty(len(x), dtype=np.int64)
    pos[order] = np.arange(len(x))
    return toks, pos


@pytest.mark.parametrize("n,scale,t,top_p", [(300, 8.0, 1.0, 1.0), (3000, 30.0, 1.0, 0.9),
                                             (151936, 12.0, 0.8, 1.0), (151936, 30.0, 1.0, 0.9)])
def test_reference_rounding_moves_large_vocabulary_draws_to_neighbours(orc, n, scale, t, top_p):
    """On small vocabularies the reference's f32 steps draw what exact
    arithmetic draws; over 151,936 entries its sequential f32 softmax sum
    drops the terms below half an ulp of the running sum, so its draws land a
    few positions away (index order without filters, rank order with top_p),
    never far. The device sampler is checked against the exact steps there."""
    x = _logits(n, 5, scale)
    s = orc.Sampler(t, 0, top_p, 77)
    ref = [s.sample(x) for _ in range(64)]
    us = (py_stdrng_u32(77, 64) >> 8).astype(np.float64) * 2.0 ** -24
    exact, pos = _exact_draws(x, t, top_p, us)
    dist = [abs(int(pos[a]) - int(pos[b])) for a, b in zip(ref, exact)]
    if n <= 3000:
        assert ref == exact
    else:
        assert max(dist) <= 64 and sum(d > 0 for d in dist) > 0
