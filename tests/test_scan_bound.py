"""The chunk-skipping lower bound of the main scan pass, restated on the CPU.

The main pass drops a (pair, 32-vector chunk) when the chunk's factor range proves that
every fp32 lower bound it would compute is >= T1 (``range_at_least`` and ``ip_term_bound``
in ``csrc/kernels_scan.cuh``). These tests evaluate the lower bound exactly as the kernel
does (numpy float32, one rounding per operation, reference
``src/search/filter_kernels.cuh:693-696``) for random and adversarial chunks and check that
the bound never drops a chunk holding a vector with low < T, and that it does drop far
chunks (it is not vacuous).
"""
import numpy as np
import pytest

f32 = np.float32


def low_f32(f_add, f_rescale, f_error, ip, width, k1, g):
    """fp32 lower bound of the scan kernel for integer inner products ip."""
    gerr = np.sqrt(np.maximum(f32(g), f32(0)), dtype=np.float32)
    ip1 = (f32(width) * ip.astype(np.float32)).astype(np.float32) + f32(0)
    t = (ip1 + f32(k1)).astype(np.float32)
    a = (f_add + f32(g)).astype(np.float32)
    b = (f_rescale * t).astype(np.float32)
    e = (f_error * gerr).astype(np.float32)
    return ((a + b).astype(np.float32) - e).astype(np.float32)


def ip_term_bound(pos, neg, width, k1):
    hi = (f32(width) * f32(pos)) + f32(0) + f32(k1)
    lo = (f32(width) * f32(neg)) + f32(0) + f32(k1)
    return max(abs(f32(hi)), abs(f32(lo)))


def range_at_least(f_add, f_rescale, f_error, g, M, T):
    gerr = float(np.sqrt(np.maximum(f32(g), f32(0)), dtype=np.float32))
    mn = float(np.min(f_add))
    mx = float(np.max(np.abs(f_add)))
    r = float(np.max(np.abs(f_rescale))) * float(M)
    e = float(np.max(np.abs(f_error))) * gerr
    L = (mn + float(g)) - r - e
    S = mx + abs(float(g)) + r + e
    return L - 2.0 ** -20 * S >= float(T)


def _chunk(rng, scale):
    n = 32
    f_add = (rng.standard_normal(n) * scale[0] + scale[1]).astype(np.float32)
    f_rescale = (-np.abs(rng.standard_normal(n)) * scale[2]).astype(np.float32)
    f_error = (np.abs(rng.standard_normal(n)) * scale[3]).astype(np.float32)
    return f_add, f_rescale, f_error


@pytest.mark.parametrize("seed", range(6))
def test_bound_never_drops_a_candidate(seed):
    rng = np.random.default_rng(seed)
    dropped = 0
    for trial in range(3000):
        scale = (rng.uniform(0.01, 50), rng.uniform(-100, 200), rng.uniform(0.01, 5),
                 rng.uniform(0, 3))
        f_add, f_rescale, f_error = _chunk(rng, scale)
        D = 128
        qint = rng.integers(-128, 128, D)
        pos, neg = int(qint[qint > 0].sum()), int(qint[qint < 0].sum())
        width = f32(rng.uniform(1e-3, 0.2))
        k1 = f32(rng.uniform(-50, 50))
        g = f32(rng.uniform(0, 300))
        M = ip_term_bound(pos, neg, width, k1)
        # the reachable inner products, endpoints included
        ip = rng.integers(neg, pos + 1, 32)
        ip[:2] = [neg, pos]
        lows = low_f32(f_add, f_rescale, f_error, ip, width, k1, g)
        # thresholds straddling the smallest low, where rounding matters most
        m = float(lows.min())
        for T in (np.nextafter(f32(m), f32(np.inf)), f32(m), np.nextafter(f32(m), f32(-np.inf)),
                  f32(m - 1.0), f32(rng.uniform(-100, 300))):
            if range_at_least(f_add, f_rescale, f_error, g, M, T):
                dropped += 1
                assert np.all(lows >= T), (trial, T, lows.min())
    assert dropped > 0


def test_bound_drops_far_chunks():
    """A query far from a compact cluster: the whole chunk is provably above T."""
    rng = np.random.default_rng(7)
    D = 128
    q = rng.standard_normal(D).astype(np.float32) * 1.0
    width = f32(np.abs(q).max() / 127)
    qint = np.clip(np.rint(q / width), -128, 127).astype(np.int64)
    k1 = f32(-0.5 * q.sum())
    pos, neg = int(qint[qint > 0].sum()), int(qint[qint < 0].sum())
    M = ip_term_bound(pos, neg, width, k1)
    f_add = (6.0 + rng.standard_normal(32)).astype(np.float32)
    f_rescale = (-1.25 + 0.05 * rng.standard_normal(32)).astype(np.float32)
    f_error = (0.7 + 0.05 * rng.standard_normal(32)).astype(np.float32)
    g = f32(102.0)  # squared distance to the far centroid
    assert range_at_least(f_add, f_rescale, f_error, g, M, f32(12.0))
    assert not range_at_least(f_add, f_rescale, f_error, f32(6.0), M, f32(12.0))


@pytest.mark.parametrize("seed", range(4))
def test_bound_tight_chunks(seed):
    """Equal factors and inner products at the end of their range: the lows sit on the
    bound itself, so only the rounding margin keeps the test sound."""
    rng = np.random.default_rng(100 + seed)
    dropped = 0
    for trial in range(4000):
        D = 128
        qint = rng.integers(-128, 128, D)
        pos, neg = int(qint[qint > 0].sum()), int(qint[qint < 0].sum())
        width = f32(rng.uniform(1e-3, 0.2))
        k1 = f32(rng.uniform(-50, 50))
        g = f32(rng.uniform(0, 300))
        M = ip_term_bound(pos, neg, width, k1)
        f_add = np.full(32, f32(rng.uniform(-100, 300)), np.float32)
        fr = f32(rng.uniform(0.01, 5))
        f_error = np.full(32, f32(rng.uniform(0, 3)), np.float32)
        hi = f32(f32(width * f32(pos)) + f32(k1))
        lo = f32(f32(width * f32(neg)) + f32(k1))
        # the end of the ip range where |t| = M, and f_rescale * t = -|f_rescale| * M there
        ip_end, t_end = (pos, hi) if abs(hi) >= abs(lo) else (neg, lo)
        assert abs(t_end) == M
        f_rescale = np.full(32, f32(-fr if t_end > 0 else fr), np.float32)
        ip = np.full(32, ip_end)
        lows = low_f32(f_add, f_rescale, f_error, ip, width, k1, g)
        m = float(lows.min())
        gerr = float(np.sqrt(g, dtype=np.float32))
        L = float(f_add[0]) + float(g) - float(fr) * float(M) - float(f_error[0]) * gerr
        S = abs(float(f_add[0])) + float(g) + float(fr) * float(M) + float(f_error[0]) * gerr
        # the lows sit on the bound up to rounding
        assert abs(L - m) <= 2.0 ** -21 * S
        for T in (np.nextafter(f32(m), f32(np.inf)), f32(m), np.nextafter(f32(m), f32(-np.inf)),
                  f32(L - 2.0 ** -19 * S)):
            if range_at_least(f_add, f_rescale, f_error, g, M, T):
                dropped += 1
                assert np.all(lows >= T), (trial, T, lows.min())
    assert dropped > 0


def lut_bound(lut_f16, k1):
    """The LUT estimator's bound M (lut_build_kernel): Hi / Lo the sums of each group's
    largest / smallest entry, A the sum of the largest magnitudes; rounded outwards."""
    e = lut_f16.astype(np.float64)                       # (D / 4, 16), exact halves
    hi, lo = e.max(1).sum(), e.min(1).sum()
    A = np.maximum(e.max(1), -e.min(1)).sum()
    span = max(np.nextafter(hi + float(k1), np.inf), -np.nextafter(lo + float(k1), -np.inf))
    m = (span + A * 2.0 ** -16) * (1 + 2.0 ** -22)
    return np.nextafter(np.float32(m), np.float32(np.inf)) if np.float32(m) < m else np.float32(m)


@pytest.mark.parametrize("D", [128, 192, 768])
def test_lut_bound_covers_every_code(D):
    """|fl(ip1 + k1)| <= M for the LUT estimator, with ip1 from the oracle's fp32 table sums
    (cora_oracle_ip_lut), on random codes and on the codes that select each group's largest
    or smallest entry (the ends of the range), for queries of several scales."""
    import py_oracle as po
    rng = np.random.default_rng(D)
    W = D // 32
    for trial in range(40):
        qr = (rng.standard_normal(D) * 10.0 ** rng.uniform(-3, 2)).astype(np.float32)
        lut = np.empty(D * 4, np.uint16)
        po.lib().cora_oracle_query_lut(qr, D, lut)
        tab = lut.view(np.float16).reshape(D // 4, 16)
        k1 = np.float32(np.float32(qr.astype(np.float64).sum()) * np.float32(-0.5))
        M = lut_bound(tab, k1)
        codes = [rng.integers(0, 2 ** 32, W, dtype=np.uint64).astype(np.uint32) for _ in range(30)]
        for pick in (np.argmax, np.argmin):  # the extreme pattern of every group
            pats = pick(tab.astype(np.float32), axis=1)
            words = np.zeros(W, np.uint32)
            for g, pval in enumerate(pats):
                w, n = divmod(g, 8)
                words[w] |= np.uint32(int(pval) << (28 - 4 * n))
            codes.append(words)
        for words in codes:
            ip1 = np.float32(po.lib().cora_oracle_ip_lut(np.ascontiguousarray(words), lut, D))
            t = np.float32(ip1 + k1)
            assert abs(t) <= M, (trial, t, M)
