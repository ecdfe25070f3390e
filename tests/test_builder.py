"""CPU tests: the torch index builder (coraanns_b200.builder) pinned against the reference's
own quantizer, rabitqlib::ivf::IVF::construct(faster = true) (third_party/rabitq/include/
rabitqlib/index/ivf/ivf.hpp:221-303, quantizer rabitq_impl.hpp:76-137 and 379-500).

The reference draws its rotation and its "faster" ex-code rescale constant t_const from an
unseeded random source, so the comparison quantises the same vectors against the reference's
own choices: its rotator and rotated centroids are read back from the index file it wrote,
and t_const is recovered from its ex codes (every code u_i = floor(t o_i + 1e-5), clipped
at 127, confines t to an interval; the intersection over all dimensions of all vectors is
narrow, and any t inside it reproduces every code).
"""
from __future__ import annotations

import numpy as np
import pytest

import py_oracle as po

pytestmark = pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")


def _data(n, dim, nlist, seed):
    rng = np.random.default_rng(seed)
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    lab = rng.integers(0, nlist, n)
    base = (centres[lab] + 0.25 * rng.normal(size=(n, dim))).astype(np.float32)
    return base, centres, lab.astype(np.uint32)


def _unpack_bits(sd):
    """n x D bool 1-bit codes in cluster order from the adapter's word-major layout."""
    D, n = int(sd["D"]), int(sd["num"])
    W = D // 32
    bits = np.zeros((n, D), bool)
    start = 0
    for nc in sd["sizes"].astype(np.int64):
        words = sd["short_data"][start * W:(start + nc) * W].reshape(W, nc).T  # nc x W
        for w in range(W):
            for b in range(32):
                bits[start:start + nc, 32 * w + b] = (words[:, w] >> np.uint32(31 - b)) & 1
        start += nc
    return bits


def _residuals(data_sorted, rot, crot_rows):
    """Rotated residuals r = x P - c' (fp64 product rounded to fp32, as the builder forms
    them), their normalised magnitudes o = |r| / ||r||, and the components whose sign the
    last bits decide: the reference forms x P in fp32 sums, whose error grows with the row's
    norm (not with the component), so |r| within 2^-18 of max(||x||, |c'|) counts as zero."""
    xr = (data_sorted.astype(np.float64) @ rot.astype(np.float64)).astype(np.float32)
    r = xr.astype(np.float64) - crot_rows.astype(np.float64)
    scale = np.maximum(np.linalg.norm(data_sorted.astype(np.float64), axis=1, keepdims=True),
                       np.abs(crot_rows).astype(np.float64))
    near_zero = np.abs(r) <= 2.0 ** -18 * scale
    return r, np.abs(r) / np.linalg.norm(r, axis=1, keepdims=True), near_zero


def _recover_t(o, bits, u):
    """The t_const most consistent with the reference's ex codes: each raw code c (the
    stored code, un-flipped for negative components) gives c <= t o + 1e-5 < c + 1 (no
    upper bound at 127); the fp32 residuals of the reference and the fp64-rounded ones
    here differ in the last bits, so a handful of constraints on floor boundaries can
    conflict: t minimises the violations over the narrow band where the bounds meet."""
    raw = np.where(bits, u, 127 - u).astype(np.float64)
    ok = o > 1e-6
    lo = np.where(ok, (raw - 1e-5) / np.where(ok, o, 1), -np.inf).ravel()
    hi = np.where(ok & (raw < 127), (raw + 1 - 1e-5) / np.where(ok, o, 1), np.inf).ravel()
    a, b = hi.min(), lo.max()
    grid = np.linspace(min(a, b) - 1e-3, max(a, b) + 1e-3, 101)
    viol = np.array([((lo > t) | (hi <= t)).sum() for t in grid])
    return float(grid[int(np.argmin(viol))]), int(viol.min())


def _decode(sd, n, D):
    u = np.zeros((n, D), np.uint8)
    codes = sd["long_codes"].reshape(n, D * 7 // 8)
    for i in range(n):
        po.lib().cora_oracle_decode_ex7(np.ascontiguousarray(codes[i]), D, u[i])
    return u


@pytest.mark.parametrize("n,dim,nlist,seed,metric", [(3000, 96, 16, 41, 0), (1200, 200, 8, 42, 0),
                                                     (2000, 128, 8, 43, 1)])
def test_builder_matches_reference_faster_quantizer(tmp_path, n, dim, nlist, seed, metric):
    base, centres, lab = _data(n, dim, nlist, seed)
    if metric == 1:  # inner product on unit vectors
        base /= np.linalg.norm(base, axis=1, keepdims=True)
    path = tmp_path / "ref.index"
    po.ref_build_index(path, base, centres, lab, total_bits=8, faster=True, metric_ip=metric == 1)
    ref = po.search_data(po.read_ivf_file(path))
    assert ref["metric"] == metric
    D = int(ref["D"])
    ref_bits = _unpack_bits(ref)
    ref_u = _decode(ref, n, D)
    order = ref["ids"].astype(np.int64)
    assert np.array_equal(order, np.argsort(lab, kind="stable")), "cluster order of the ids"
    r, o, near_zero = _residuals(base[order], ref["rotator"], ref["centroids"][lab[order]])
    t, conflicts = _recover_t(o, ref_bits, ref_u.astype(np.int64))
    assert conflicts <= 1e-4 * n * D, conflicts

    from coraanns_b200 import builder
    mine = builder.build_index(base, centres, lab, rotator=ref["rotator"],
                               rotated_centroids=ref["centroids"], t_const=t, metric=metric)
    assert np.array_equal(mine["ids"], ref["ids"])
    assert np.array_equal(mine["sizes"], ref["sizes"])
    # 1-bit codes: identical except where a residual component lies within rounding of zero
    bit_diff = _unpack_bits(mine) != ref_bits
    assert not (bit_diff & ~near_zero).any(), np.argwhere(bit_diff & ~near_zero)[:5]
    assert bit_diff.sum() <= 1e-4 * n * D
    # 7-bit ex codes: identical except on a floor boundary (differing by one, within 1e-3 of
    # t o + 1e-5 being an integer: o's last bits times t ~ 500) or where the sign flipped
    # (the stored code is mirrored)
    u = _decode(mine, n, D)
    diff = u != ref_u
    assert diff.sum() <= 2e-4 * n * D, diff.sum()
    v = t * o + 1e-5
    floor_edge = np.abs(v - np.round(v)) < 1e-3
    assert not (diff & ~(near_zero | floor_edge)).any(), np.argwhere(diff & ~(near_zero | floor_edge))[:5]
    assert np.abs(u.astype(np.int64) - ref_u)[diff & ~near_zero].max(initial=0) <= 1
    # factors (fp32 Eigen sums in the reference, fp64 rounded once here) of the vectors with
    # identical codes: within 2e-6 of the vector's distance scale max(|factor|, ||r||^2)
    same = ~(diff | bit_diff).any(1)
    assert same.mean() >= 0.99
    l2 = (r * r).sum(1)[:, None]
    if metric == 1:  # the factors' scale includes the constant 1 of 1 - <q, x>
        l2 = np.maximum(l2, 1.0)
    for key in ("short_factors", "ex_factors"):
        a, b = mine[key].astype(np.float64), ref[key].astype(np.float64)
        err = np.abs(a - b) / np.maximum(np.abs(b), l2)
        assert err[same].max() <= 2e-6, (key, err[same].max(0))
