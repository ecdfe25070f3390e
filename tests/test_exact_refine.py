"""Exact FP32 refinement (the reference's HybridIndex::enable_exact_refine, hybrid.cuh:171-178;
the refine step cpu_refinement.cpp:168-181): every candidate's distance is the exact squared
L2 distance between the raw query and its base row (by original id); candidates whose id is
outside the base, or all of them when the base dimension differs, are dropped.

CPU: the oracle's exact mode against a numpy restatement. GPU: the engine through the C ABI
against the oracle, bit for bit.
"""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

import py_oracle as po
from conftest import GOLDEN, regen_base


def exact_dist(q, b):
    """fp32 of the fp64 fma chain acc = fma(d, d, acc) over d = q_j - b_j (in fp64),
    j ascending; each fma is rounded once (exact rational arithmetic, then to float64)."""
    acc = 0.0
    for qj, bj in zip(q.tolist(), b.tolist()):
        d = qj - bj  # fp32 values: their fp64 difference rounds like the kernels' dsub
        acc = float(Fraction(d) * Fraction(d) + Fraction(acc))
    return np.float32(acc)


def _demo():
    z = np.load(GOLDEN / "demo.npz")
    base = regen_base(z["meta"], z["gen"])
    return z, base


def test_oracle_exact_distances_and_order():
    z, base = _demo()
    o = po.oracle_from_file(GOLDEN / "demo.index")
    q = z["queries"][:12]
    o.set_exact_base(base)
    d, i = o.search(q, 10, 8)
    for n in range(q.shape[0]):
        for j in range(10):
            if d[n, j] == np.finfo(np.float32).max:
                continue
            assert d[n, j] == exact_dist(q[n], base[i[n, j]])
        keys = list(zip(d[n].tolist(), i[n].tolist()))
        assert keys == sorted(keys)
    # the exact distances rank at least as well as the ex-code estimates against the truth
    o.set_exact_base(None)
    d_est, i_est = o.search(q, 10, 8)
    gt = z["gt_ids"][:12, :10]
    hits = lambda ids: sum(len(set(a) & set(b)) for a, b in zip(ids.tolist(), gt.tolist()))
    assert hits(i) >= hits(i_est)


def test_oracle_exact_rows_outside_the_base_are_dropped():
    z, base = _demo()
    o = po.oracle_from_file(GOLDEN / "demo.index")
    q = z["queries"][:12]
    rows = base.shape[0] // 2
    o.set_exact_base(base[:rows])
    det = o.search(q, 10, 8, with_details=True)
    ok = det["dist"] != np.finfo(np.float32).max
    assert ok.any()
    assert (det["ids"][ok] < rows).all()
    # a base of another dimension drops every candidate
    o.set_exact_base(base[:, :-1])
    d, i = o.search(q, 10, 8)
    assert (d == np.finfo(np.float32).max).all() and (i == 0).all()


@pytest.mark.gpu
def test_gpu_exact_refine_matches_oracle():
    import coraanns_b200 as cb
    z, base = _demo()
    q = z["queries"][:40]
    o = po.oracle_from_file(GOLDEN / "demo.index")
    e = cb.HybridIndex(0)
    e.load_index_file(str(GOLDEN / "demo.index"))
    e.prepare_workspace(len(q), 10, 8)
    for b in (base, base[: base.shape[0] // 2], base[:, :-1], None):
        e.enable_exact_refine(b)
        o.set_exact_base(b)
        for graphs in (1, 0):
            e.set_tuning("search_graphs", graphs)
            e.reset_buffer(q)
            d, i = e.search(q, 10, 8)
            rd, ri = o.search(q, 10, 8)
            assert d.tobytes() == rd.tobytes()
            assert np.array_equal(i, ri)
    e.close()
