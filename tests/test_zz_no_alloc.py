"""cora_probe_noalloc: coarse probing that allocates nothing (static per-device scratch).

Compared through the C ABI with the probe list the regular search entry point computes
(cora_search, then cora_debug_copy arrays 1 and 2) on two calls in a row, with device free
memory unchanged across the calls. Collected last on purpose; it also passes alone.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb():
    import coraanns_b200
    return coraanns_b200


def _synthetic(n, dim, nlist, nq, seed, same_centre=False):
    from coraanns_b200 import builder
    rng = np.random.default_rng(seed)
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    if same_centre:  # every centroid equal: the guarded band overflows -> exact fallback
        centres = np.repeat(centres[:1], nlist, 0)
    lab = np.arange(n) % nlist
    data = (centres[lab] + 0.3 * rng.normal(size=(n, dim))).astype(np.float32)
    q = (centres[rng.integers(0, nlist, nq)] + 0.3 * rng.normal(size=(nq, dim))).astype(np.float32)
    return builder.build_index(data, centres, lab, seed=seed), q


def _search_probes(cb, load, q, nprobe):
    """Probe ids/distances of the existing entry point (cora_search)."""
    e = cb.HybridIndex(0)
    load(e)
    e.prepare_workspace(q.shape[0], 10, nprobe)
    e.reset_buffer(q)
    e.search(q, 10, nprobe)
    out = e.debug("probe_ids", q.shape[0], nprobe), e.debug("probe_g", q.shape[0], nprobe)
    e.close()
    return out


def _noalloc_twice(cb, load, q, nprobe):
    import torch
    e = cb.HybridIndex(0)
    load(e)
    dq = torch.from_numpy(q).cuda()
    ids = torch.full((q.shape[0], nprobe), -1, dtype=torch.int32, device="cuda")
    dist = torch.full((q.shape[0], nprobe), float("nan"), dtype=torch.float32, device="cuda")
    results = []
    torch.cuda.synchronize()
    free_before = None
    for call in range(2):
        ids.fill_(-1)
        dist.fill_(float("nan"))
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
        e.probe_noalloc(dq.data_ptr(), q.shape[0], nprobe, ids.data_ptr(), dist.data_ptr())
        e.probe_noalloc_status()  # synchronises; raises if a device-side wait gave up
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before, "the call allocated device memory"
        results.append((ids.cpu().numpy().copy(), dist.cpu().numpy().copy()))
    e.close()
    return results


def _compare(cb, load, q, nprobe):
    want_ids, want_g = _search_probes(cb, load, q, nprobe)
    for got_ids, got_g in _noalloc_twice(cb, load, q, nprobe):
        # the same kernels on the same inputs: identical bytes, not merely close values
        assert np.array_equal(got_ids, want_ids)
        assert got_g.tobytes() == want_g.tobytes()


def test_noalloc_probe_matches_search_golden(cb):
    with np.load(GOLDEN / "demo.npz") as z:
        q = z["queries"]
    _compare(cb, lambda e: e.load_index_file(str(GOLDEN / "demo.index")), q, 8)


@pytest.mark.parametrize("same_centre", [False, True])
def test_noalloc_probe_matches_search_synthetic(cb, same_centre):
    sd, q = _synthetic(32768, 128, 2048, 384, seed=21, same_centre=same_centre)
    _compare(cb, lambda e: e.load_search_data(sd), q, 32)


def test_noalloc_probe_block_selection(cb):
    """nprobe > 32: one block-wide selection per query (no warp pass, no fallback list)."""
    sd, q = _synthetic(32768, 128, 2048, 256, seed=33)
    _compare(cb, lambda e: e.load_search_data(sd), q, 64)


def test_noalloc_probe_matches_oracle(cb):
    """The probe list against the CPU oracle's exact top-nprobe on a golden index."""
    import py_oracle as po
    import torch
    with np.load(GOLDEN / "d96.npz") as z:
        q = z["queries"]
    path = GOLDEN / "d96.index"
    oracle = po.oracle_from_file(path)
    want_ids, want_g = oracle.probe(oracle.rotate(q), 6)
    e = cb.HybridIndex(0)
    e.load_index_file(str(path))
    dq = torch.from_numpy(q).cuda()
    ids = torch.empty((q.shape[0], 6), dtype=torch.int32, device="cuda")
    dist = torch.empty((q.shape[0], 6), dtype=torch.float32, device="cuda")
    e.probe_noalloc(dq.data_ptr(), q.shape[0], 6, ids.data_ptr(), dist.data_ptr())
    e.probe_noalloc_status()
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert dist.cpu().numpy().tobytes() == want_g.tobytes()
    e.close()


def test_noalloc_probe_rejects(cb):
    import torch
    limit = cb.probe_noalloc_scratch_limit()
    assert limit == 16 << 20
    sd, q = _synthetic(8192, 128, 2048, 2000, seed=5)
    e = cb.HybridIndex(0)
    dq = torch.from_numpy(q).cuda()
    ids = torch.empty((q.shape[0], 8), dtype=torch.int32, device="cuda")
    dist = torch.empty((q.shape[0], 8), dtype=torch.float32, device="cuda")
    with pytest.raises(cb.LogicError):  # no index yet
        e.probe_noalloc(dq.data_ptr(), 4, 8, ids.data_ptr(), dist.data_ptr())
    e.load_search_data(sd)
    # 2000 queries x (rotated query + planes + 2048 approximate distances) > 16 MiB
    with pytest.raises(cb.InvalidArgument, match="static limit"):
        e.probe_noalloc(dq.data_ptr(), 2000, 8, ids.data_ptr(), dist.data_ptr())
    with pytest.raises(cb.InvalidArgument):
        e.probe_noalloc(dq.data_ptr(), 4, 2049, ids.data_ptr(), dist.data_ptr())
    with pytest.raises(cb.InvalidArgument):
        e.probe_noalloc(dq.data_ptr(), 0, 8, ids.data_ptr(), dist.data_ptr())
    # a call within the limit still works after the rejected ones
    e.probe_noalloc(dq.data_ptr(), 16, 8, ids.data_ptr(), dist.data_ptr())
    torch.cuda.synchronize()
    assert (ids[:16] >= 0).all() and (ids[:16] < 2048).all()
    e.close()
