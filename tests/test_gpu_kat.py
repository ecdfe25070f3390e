"""GPU ports of the reference's own GPU tests (tests/gpu_*.cpp of the reference project),
minus the checks that only concern its host ring buffer."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import kat_fixture

pytestmark = pytest.mark.gpu
FLT_MAX = np.finfo(np.float32).max


@pytest.fixture(scope="module")
def cb():
    import coraanns_b200
    return coraanns_b200


def _init(cb, sd, nq, k, nprobe, capacity=None, spill=None, vanguard=5):
    e = cb.HybridIndex(0)
    if capacity is not None:
        e.set_queue_capacity(capacity)
    if spill is not None:
        e.set_queue_spill_capacity(spill)
    e.set_vanguard_size(vanguard)
    e.set_candidate_stats(True)
    e.load_search_data(sd)
    e.prepare_workspace(nq, k, nprobe)
    return e


def _check(e, sd, q, expected, k, chunk, batch_q=4, count=32768):
    nq = len(q)
    ids = np.zeros((nq, k), np.uint32)
    dist = np.zeros((nq, k), np.float32)
    for b in range(0, nq, chunk):
        n = min(chunk, nq - b)
        e.reset_buffer(q[b:b + n])
        d, i = e.search(q[b:b + n], k, 8, batch_q=batch_q)
        ids[b:b + n], dist[b:b + n] = i, d
        # gpu_cpu_ring_queue_test.cpp:78-82
        assert e.get_last_submitted_count() == n * count, "dropped or duplicated candidates"
        assert e.get_last_refined_count() == n * count
    for a in range(nq):
        assert np.array_equal(np.sort(ids[a]), expected), "exact nearest ids changed"
        qn = np.float32(0)
        for d_ in range(q.shape[1]):
            qn = np.float32(qn + q[a, d_] * q[a, d_])
        exp = sd["ex_factors"][ids[a], 0] + qn
        assert np.abs(dist[a] - exp).max() < 1e-4, "payload distances"


@pytest.mark.parametrize("capacity", [8192, 262144])
@pytest.mark.parametrize("vanguard", [0, 5])
def test_ring_queue_kat(cb, capacity, vanguard):
    """gpu_cpu_ring_queue_test.cpp:100-124: exact ids/distances, repeated searches, chunks."""
    sd, q, expected = kat_fixture()
    e = _init(cb, sd, 5, 100, 8, capacity=capacity, spill=262144, vanguard=vanguard)
    for _ in range(3):
        _check(e, sd, q, expected, 100, 5)
        assert e.get_last_spilled_count() == 0
        _check(e, sd, q, expected, 100, 2)
    e.close()


def test_partial_chunk_small_capacity(cb):
    """gpu_cpu_ring_queue_test.cpp:125-139 (1032 vectors, k = 10, tiny capacity)."""
    sd, q, expected = kat_fixture(count=1032, topk=10)
    for capacity in (32, 8192):
        e = _init(cb, sd, 5, 10, 8, capacity=capacity, spill=8192, vanguard=0)
        for _ in range(4):
            _check(e, sd, q, expected, 10, 5, count=1032)
        e.close()


@pytest.mark.parametrize("batch_q", [1, 2, 3, 5, 6])
def test_batch_q_values(cb, batch_q):
    """gpu_cpu_ring_queue_test.cpp:140-147."""
    sd, q, expected = kat_fixture()
    e = _init(cb, sd, 5, 100, 8, capacity=8192, spill=262144)
    _check(e, sd, q, expected, 100, 5, batch_q=batch_q)
    e.close()


def test_cross_query_reuse_off(cb):
    sd, q, expected = kat_fixture()
    e = _init(cb, sd, 5, 100, 8)
    e.set_cross_query_reuse(False)
    _check(e, sd, q, expected, 100, 5)
    e.close()


def test_empty_results(cb):
    """gpu_cpu_ring_queue_test.cpp:148-167: no candidates -> FLT_MAX, repeatedly."""
    sd, q, _ = kat_fixture(f_add=FLT_MAX)
    e = _init(cb, sd, 5, 100, 8, capacity=8192, spill=1024, vanguard=0)
    for _ in range(3):
        e.reset_buffer(q)
        d, i = e.search(q, 100, 8)
        assert e.get_last_submitted_count() == 0
        assert np.all(d == FLT_MAX)
    e.close()


def test_overflow_reported_then_reset(cb):
    """gpu_cpu_ring_queue_test.cpp:180-202: exhausted capacity raises a runtime error that
    names the spill capacity, without hanging; a reset search afterwards is clean."""
    sd, q, _ = kat_fixture()
    e = _init(cb, sd, 5, 100, 8, capacity=32, spill=0, vanguard=0)
    e.reset_buffer(q)
    with pytest.raises(RuntimeError, match="spill capacity exhausted"):
        e.search(q, 100, 8)
    e.reset_buffer(q)
    e.seed_thresholds(np.full(5, -FLT_MAX, np.float32))
    e.search(q, 100, 8)
    assert e.get_last_submitted_count() == 0
    e.close()


def test_lifecycle(cb):
    """gpu_search_lifecycle_test.cpp:15-64."""
    dim, count, queries = 128, 32, 2
    q = np.zeros((queries, dim), np.float32)
    rot = np.eye(dim, dtype=np.float32)
    sd = dict(num=count, dim=dim, D=dim, nlist=1, ex_bits=7,
              centroids=np.zeros((1, dim), np.float32), rotator=rot,
              short_data=np.zeros(count * dim // 32, np.uint32),
              short_factors=np.tile(np.array([1e6, 0, 0], np.float32), (count, 1)),
              long_codes=np.zeros(count * dim * 7 // 8, np.uint8),
              ex_factors=np.zeros((count, 2), np.float32),
              ids=np.arange(count, dtype=np.uint32), sizes=np.array([count], np.uint64))
    e = cb.HybridIndex(0)
    with pytest.raises(cb.LogicError):
        e.prepare_workspace(queries, 10, 1)
    with pytest.raises(cb.LogicError):
        e.reset_buffer(q)
    with pytest.raises(cb.LogicError):
        e.search(q, 10, 1)
    e.load_search_data(sd)
    with pytest.raises(cb.LogicError):
        e.load_search_data(sd)  # index already loaded
    e.set_queue_capacity(32)
    e.set_queue_spill_capacity(1024)
    e.set_vanguard_size(0)
    with pytest.raises(cb.LogicError):
        e.prepare_workspace(65536, 10, 1)
    e.prepare_workspace(queries, 10, 1)
    with pytest.raises(cb.LogicError):
        e.set_queue_capacity(64)  # after prepare_workspace
    q3 = np.zeros((queries + 1, dim), np.float32)
    with pytest.raises(cb.LogicError):
        e.reset_buffer(q3)
    with pytest.raises(cb.LogicError):
        e.search(q3, 10, 1)
    with pytest.raises(cb.LogicError):
        e.search(q, 11, 1)
    with pytest.raises(cb.LogicError):
        e.search(q, 10, 2)
    with pytest.raises(cb.LogicError):
        e.search(q, 10, 1, batch_q=7)
    for it in range(3):
        e.reset_buffer(q)
        e.seed_thresholds(np.full(queries, -1, np.float32))
        d, i = e.search(q, 10, 1)
        assert np.all(d == FLT_MAX)
        e.free_workspace()
        e.free_workspace()
        with pytest.raises(cb.LogicError):
            e.reset_buffer(q)
        e.set_vanguard_size(1 if it == 0 else 0)
        e.prepare_workspace(queries, 10, 1)
    e.close()


def test_highk_vanguard_on_off(cb):
    """gpu_cpu_highk_vanguard_test.cpp:146-183: k up to 1024, vanguard on/off and chunked
    searches return identical ids and distances; ids are the k smallest f_add_ex."""
    sd, q, _ = kat_fixture(topk=1024)
    e = _init(cb, sd, 5, 1024, 8, vanguard=5)
    for k in (10, 50, 100, 200, 500, 512, 513, 1000, 1024):
        e.set_vanguard_size(0)
        e.reset_buffer(q)
        d0, i0 = e.search(q, k, 8)
        expected = np.sort(np.argsort(sd["ex_factors"][:, 0], kind="stable")[:k]).astype(np.uint32)
        for a in range(5):
            assert np.array_equal(np.sort(i0[a]), expected)
        e.set_vanguard_size(5)
        for _ in range(2):
            e.reset_buffer(q)
            d5, i5 = e.search(q, k, 8)
            assert np.array_equal(i5, i0) and d5.tobytes() == d0.tobytes()
            parts = []
            for b in (0, 2, 4):
                e.reset_buffer(q[b:b + 2])
                parts.append(e.search(q[b:b + 2], k, 8))
            assert np.array_equal(np.concatenate([p[1] for p in parts]), i0)
            assert np.concatenate([p[0] for p in parts]).tobytes() == d0.tobytes()
    e.close()
