"""GPU parity: the CUDA path through the C ABI against the oracle, bit for bit.

Each test compares the pipeline stage by stage (rotated queries, query scalars and
bit-planes, probe lists, seeded thresholds, candidate counts and sets, final distances and
ids), so the first failing assertion names the first diverging kernel.
"""
from __future__ import annotations

import numpy as np
import pytest

import py_oracle as po
from conftest import GOLDEN_NAMES

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb():
    import coraanns_b200
    return coraanns_b200


# forms of the search contract: "" integer estimator + the reference's refinement (the
# default), "T" full-code refinement, "L" fp16-LUT estimator (the golden keys' suffixes)
FORMS = {"": dict(), "T": dict(full_code=True), "L": dict(lut=True)}


def _engine(cb, path=None, sd=None, nq=1, k=10, nprobe=1, vanguard=5, mode="lows",
            full_code=False, lut=False):
    e = cb.HybridIndex(0)
    e.set_vanguard_size(vanguard)
    e.set_refine_full_code(full_code)
    e.set_ip_kernel_type(cb.KernelType.Lut4Bit if lut else cb.KernelType.Bitwise)
    if mode == "rescan":
        e.set_vanguard_lows_budget(0)
    if mode == "blocksel":  # every pair / query through the block-wide selections
        e.set_tuning("warp_select_limit", 0)
        e.set_tuning("topk_warp_limit", 0)
    if mode == "tightsel":  # the warp selections hand most pairs / queries over
        e.set_tuning("warp_select_limit", 8)
        e.set_tuning("topk_warp_limit", 4)
    if path is not None:
        e.load_index_file(path)
    else:
        e.load_search_data(sd)
    e.prepare_workspace(nq, k, nprobe)
    return e


def _check_stages(e, q, k, nprobe, ref, tag):
    nq = q.shape[0]
    if "qr" in ref:
        assert e.debug("rotated", nq).tobytes() == ref["qr"].tobytes(), f"{tag}: rotation"
    if "scalars" in ref:
        assert e.debug("scalars", nq).tobytes() == ref["scalars"].astype(np.float32).tobytes(), \
            f"{tag}: query scalars"
    if "planes" in ref:
        got = e.debug("planes", nq)
        W = ref["planes"].shape[2]
        assert np.array_equal(got[:, :, :W], ref["planes"]), f"{tag}: query bit-planes"
        assert not got[:, :, W:].any(), f"{tag}: padding planes"
    assert np.array_equal(e.debug("probe_ids", nq, nprobe), ref["probe_ids"]), f"{tag}: probes"
    assert e.debug("probe_g", nq, nprobe).tobytes() == ref["probe_g"].tobytes(), f"{tag}: probe g"
    assert e.debug("thresholds1", nq).tobytes() == ref["thresholds1"].tobytes(), f"{tag}: T1"
    assert np.array_equal(e.debug("cand_count", nq).astype(np.uint64), ref["cand_count"]), \
        f"{tag}: candidate counts"


@pytest.mark.parametrize("loader,mode,sfx", [
    ("file", "lows", ""), ("raw", "lows", ""), ("file", "rescan", ""),
    ("file", "blocksel", ""), ("raw", "tightsel", ""),
    ("file", "lows", "T"), ("raw", "rescan", "T"),
    ("file", "lows", "L"), ("raw", "rescan", "L"), ("file", "tightsel", "L")])
@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_golden_parity(cb, golden, name, loader, mode, sfx):
    """Every stage and the results against the committed oracle outputs, in each form of
    the contract (integer estimator + the reference's refinement, full-code refinement,
    fp16-LUT estimator)."""
    path, z = golden[name]
    q = z["queries"]
    grid = z["grid"]
    kmax, npmax = int(grid[:, 0].max()), int(grid[:, 1].max())
    if loader == "file":
        e = _engine(cb, path=path, nq=len(q), k=kmax, nprobe=npmax, mode=mode, **FORMS[sfx])
    else:
        e = _engine(cb, sd=po.search_data(po.read_ivf_file(path)), nq=len(q), k=kmax,
                    nprobe=npmax, mode=mode, **FORMS[sfx])
    assert e.get_vanguard_mode() == (0 if mode == "rescan" else 1)
    for k, nprobe, van in grid:
        k, nprobe, van = int(k), int(nprobe), int(van)
        tag = f"{name}/{loader} k{k}_np{nprobe}_v{van}"
        e.set_vanguard_size(van)
        e.reset_buffer(q)
        d, i = e.search(q, k, nprobe)
        key = f"k{k}_np{nprobe}_v{van}"
        ref = dict(qr=z["qr"], scalars=z["scalars"], planes=z["planes"],
                   probe_ids=z[f"probe_{key}"], probe_g=z[f"probeg_{key}"],
                   thresholds1=z[f"t1{sfx}_{key}"], cand_count=z[f"cand{sfx}_{key}"])
        _check_stages(e, q, k, nprobe, ref, tag)
        if sfx == "L":
            want = po.oracle_from_file(path).query_lut(z["qr"])
            assert np.array_equal(e.debug("lut", len(q)), want), f"{tag}: LUT tables"
        if int(z["metric"]) if "metric" in z else 0:  # inner product: the additive terms
            cent = po.search_data(po.read_ivf_file(path))["centroids"]
            pids = z[f"probe_{key}"]
            want = np.array([[po.lib().cora_oracle_ip_gadd(np.ascontiguousarray(z["qr"][a]),
                                                           np.ascontiguousarray(cent[c]), cent.shape[1])
                              for c in pids[a]] for a in range(len(q))], np.float32)
            assert e.debug("probe_gadd", len(q), nprobe).tobytes() == want.tobytes(), \
                f"{tag}: -<q', c'>"
        assert np.array_equal(i, z[f"ids{sfx}_{key}"]), f"{tag}: ids"
        assert d.tobytes() == z[f"dist{sfx}_{key}"].tobytes(), f"{tag}: distances"
        assert e.get_last_submitted_count() == int(z[f"cand{sfx}_{key}"].sum())
    e.close()


def _synthetic(n, dim, nlist, nq, seed, sigma=0.25, metric=0):
    from coraanns_b200 import builder
    rng = np.random.default_rng(seed)
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    lab = rng.integers(0, nlist, n)
    data = (centres[lab] + sigma * rng.normal(size=(n, dim))).astype(np.float32)
    q = (centres[rng.integers(0, nlist, nq)] + sigma * rng.normal(size=(nq, dim))).astype(np.float32)
    if metric == 1:  # inner product on unit vectors
        data /= np.linalg.norm(data, axis=1, keepdims=True)
        q /= np.linalg.norm(q, axis=1, keepdims=True)
    sd = builder.build_index(data, centres, lab, seed=seed, metric=metric)
    return sd, q


@pytest.mark.parametrize("n,dim,nlist,nq,k,nprobe,mode,sfx", [
    (60_000, 768, 64, 48, 100, 8, "lows", ""),
    (60_000, 768, 64, 48, 10, 8, "rescan", "L"),
    (200_000, 96, 256, 128, 10, 16, "lows", ""),
    (200_000, 96, 256, 128, 10, 16, "lows", "T"),
])
def test_inner_product_live_parity(cb, n, dim, nlist, nq, k, nprobe, mode, sfx):
    """Inner-product indexes (unit vectors, the reference quantizer's METRIC_IP factors):
    every stage, the additive terms -<q', c'>, candidates and results bit-exact to the oracle."""
    sd, q = _synthetic(n, dim, nlist, nq, seed=n + dim + 1, metric=1)
    o = po.OracleIndex(sd, **FORMS[sfx])
    assert o.metric == 1
    ref = o.search(q, k, nprobe, vanguard=5, with_details=True)
    e = _engine(cb, sd=sd, nq=nq, k=k, nprobe=nprobe, mode=mode, **FORMS[sfx])
    assert e.get_metric() == 1
    e.reset_buffer(q)
    d, i = e.search(q, k, nprobe)
    _check_stages(e, q, k, nprobe, ref, f"ip d{dim}")
    qr = e.debug("rotated", nq)
    cent = np.asarray(sd["centroids"], np.float32)
    want = np.array([[po.lib().cora_oracle_ip_gadd(np.ascontiguousarray(qr[a]),
                                                   np.ascontiguousarray(cent[c]), cent.shape[1])
                      for c in ref["probe_ids"][a]] for a in range(nq)], np.float32)
    assert e.debug("probe_gadd", nq, nprobe).tobytes() == want.tobytes()
    assert np.array_equal(i, ref["ids"])
    assert d.tobytes() == ref["dist"].tobytes()
    e.close()


@pytest.mark.parametrize("n,dim,nlist,nq,k,nprobe,van,mode,sfx", [
    (200_000, 96, 256, 256, 10, 16, 5, "lows", ""),
    (200_000, 96, 256, 256, 10, 16, 5, "rescan", ""),
    (200_000, 96, 256, 256, 10, 16, 5, "tightsel", ""),
    (200_000, 96, 256, 64, 100, 24, 5, "lows", ""),
    (200_000, 96, 256, 64, 100, 24, 5, "lows", "T"),
    (200_000, 96, 256, 256, 10, 16, 5, "lows", "L"),
    (200_000, 96, 256, 64, 100, 24, 5, "rescan", "L"),
    (60_000, 768, 64, 48, 10, 8, 5, "lows", ""),
    (60_000, 768, 64, 48, 10, 8, 3, "rescan", ""),
    (60_000, 768, 64, 48, 10, 8, 5, "lows", "T"),
    (60_000, 768, 64, 48, 10, 8, 5, "lows", "L"),
    (60_000, 768, 64, 48, 10, 8, 3, "rescan", "L"),
    (40_000, 150, 64, 64, 10, 8, 5, "lows", "L"),
    (40_000, 150, 64, 64, 10, 8, 5, "rescan", ""),
    (100_000, 128, 128, 300, 10, 32, 0, "lows", ""),
])
def test_live_oracle_parity_larger(cb, n, dim, nlist, nq, k, nprobe, van, mode, sfx):
    """Bit-exact parity with the oracle on indexes larger than the fixtures (more tiles per
    cluster, more pairs per item, D = 768, padded code words at D = 192), in both vanguard
    modes and every form of the contract."""
    sd, q = _synthetic(n, dim, nlist, nq, seed=n + dim)
    o = po.OracleIndex(sd, **FORMS[sfx])
    ref = o.search(q, k, nprobe, vanguard=van, with_details=True,
                   cand_cap=0)
    e = _engine(cb, sd=sd, nq=nq, k=k, nprobe=nprobe, vanguard=van, mode=mode, **FORMS[sfx])
    e.reset_buffer(q)
    d, i = e.search(q, k, nprobe)
    _check_stages(e, q, k, nprobe, ref, f"synthetic n{n} d{dim}")
    assert np.array_equal(i, ref["ids"])
    assert d.tobytes() == ref["dist"].tobytes()
    e.close()


@pytest.mark.parametrize("n,dim,nlist,nq", [
    (60_000, 96, 998, 300),    # ld = 1000, ragged row and column tiles
    (40_000, 768, 300, 131),   # 24 K chunks
    (20_000, 64, 16, 5),       # one tile, mostly out of bounds
])
def test_probe_gemm_error_within_guard(cb, n, dim, nlist, nq):
    """The tensor-core approximate distances stay inside the error bound the guarded
    selection assumes (|approx - exact| <= eps * (|q'| + max |c|)^2, eps = 2^-9), and the
    probe lists and distances equal the oracle's exact selection bit for bit."""
    sd, q = _synthetic(n, dim, nlist, nq, seed=nlist + dim)
    nprobe = min(8, nlist)
    e = _engine(cb, sd=sd, nq=nq, k=10, nprobe=nprobe)
    e.reset_buffer(q)
    e.search(q, 10, nprobe)
    approx = e.debug("approx", nq)[:, :nlist].astype(np.float64)
    qr = e.debug("rotated", nq).astype(np.float64)
    cent = np.asarray(sd["centroids"], np.float64)
    exact = ((qr[:, None, :] - cent[None, :, :]) ** 2).sum(2)
    r = np.sqrt((qr ** 2).sum(1))[:, None] + np.sqrt((cent ** 2).sum(1)).max()
    ratio = np.abs(approx - exact) / r ** 2
    assert ratio.max() <= 2.0 ** -9, ratio.max()
    ref = po.OracleIndex(sd).search(q, 10, nprobe, with_details=True)
    assert np.array_equal(e.debug("probe_ids", nq, nprobe), ref["probe_ids"])
    assert e.debug("probe_g", nq, nprobe).tobytes() == ref["probe_g"].tobytes()
    e.close()


def test_probe_ties_take_the_exact_fallback(cb):
    """Every centroid equidistant from every query: the guarded selection's candidate band
    holds all 2048 centroids (more than its buffer), so the exact path over every centroid
    runs; probes must still be the smallest cluster ids, bit for bit as the oracle."""
    from coraanns_b200 import builder
    rng = np.random.default_rng(11)
    nlist, dim, n, nq = 2048, 64, 16384, 16
    centres = np.repeat(rng.normal(size=(1, dim)).astype(np.float32), nlist, 0)
    lab = np.arange(n) % nlist
    data = (centres[lab] + 0.3 * rng.normal(size=(n, dim))).astype(np.float32)
    q = (centres[:nq] + 0.3 * rng.normal(size=(nq, dim))).astype(np.float32)
    sd = builder.build_index(data, centres, lab, seed=3)
    ref = po.OracleIndex(sd).search(q, 10, 16, vanguard=5, with_details=True)
    e = _engine(cb, sd=sd, nq=nq, k=10, nprobe=16)
    e.reset_buffer(q)
    d, i = e.search(q, 10, 16)
    _check_stages(e, q, 10, 16, ref, "ties")
    assert np.array_equal(i, ref["ids"]) and d.tobytes() == ref["dist"].tobytes()
    e.close()


def test_candidate_sets_identical(cb, golden):
    """L3: with fixed thresholds the candidate set {v : low(v) < T} is identical."""
    path, z = golden["demo"]
    q = z["queries"][:16]
    o = po.oracle_from_file(path)
    e = _engine(cb, path=path, nq=16, k=10, nprobe=8)
    t = np.full(16, 40.0, np.float32)
    e.reset_buffer(q)
    e.seed_thresholds(t)
    e.search(q, 10, 8)
    got = e.debug("cand_gids", 16)
    cap = got.shape[1]
    ref = o.search(q, 10, 8, vanguard=5, thresholds=t, with_details=True, cand_cap=cap)
    assert np.array_equal(got, ref["cand_gids"])
    e.close()


def test_device_entry_point_matches_host(cb, golden):
    """cora_search_device on device buffers returns what cora_search returns."""
    import torch
    path, z = golden["d96"]
    q = z["queries"]
    e = _engine(cb, path=path, nq=len(q), k=10, nprobe=6)
    e.reset_buffer(q)
    d_h, i_h = e.search(q, 10, 6)
    dq = torch.from_numpy(q).cuda()
    dd = torch.empty((len(q), 10), dtype=torch.float32, device="cuda")
    di = torch.empty((len(q), 10), dtype=torch.int32, device="cuda")
    e.reset_buffer(q)
    torch.cuda.synchronize()
    e.search_device(dq.data_ptr(), len(q), 10, 6, dd.data_ptr(), di.data_ptr())
    e.check_device()
    assert dd.cpu().numpy().tobytes() == d_h.tobytes()
    assert np.array_equal(di.cpu().numpy().view(np.uint32), i_h)
    e.close()


def test_search_graph_replay_matches_eager(cb, golden):
    """A search replayed from the captured CUDA graph returns what launching its kernels one
    by one returns, across shape, threshold and configuration changes (which rebuild or
    reuse the graph)."""
    path, z = golden["d96"]
    q = z["queries"]
    n = len(q)
    e = _engine(cb, path=path, nq=n, k=10, nprobe=8)
    results = {}
    for graphs in (1, 0):
        e.set_tuning("search_graphs", graphs)
        out = []
        for nq, k, npb in ((n, 10, 8), (n // 2, 5, 4), (n, 10, 8)):
            for _ in range(2):  # the second call replays the graph of the first
                e.reset_buffer(q[:nq])
                d, i = e.search(q[:nq], k, npb)
                out.append((d.tobytes(), i.tobytes()))
        e.reset_buffer(q)
        e.seed_thresholds(np.full(n, 30.0, np.float32))
        d, i = e.search(q, 10, 8)
        out.append((d.tobytes(), i.tobytes()))
        e.set_tuning("warp_select_limit", 8)
        e.reset_buffer(q)
        d, i = e.search(q, 10, 8)
        out.append((d.tobytes(), i.tobytes()))
        e.set_tuning("warp_select_limit", 256)
        e.set_refine_full_code(True)  # a configuration change: the graph is rebuilt
        e.reset_buffer(q)
        d, i = e.search(q, 10, 8)
        out.append((d.tobytes(), i.tobytes()))
        e.set_refine_full_code(False)
        e.reset_buffer(q)
        d, i = e.search(q, 10, 8)
        out.append((d.tobytes(), i.tobytes()))
        e.set_ip_kernel_type(cb.KernelType.Lut4Bit)  # another estimator: rebuilt again
        e.reset_buffer(q)
        d, i = e.search(q, 10, 8)
        out.append((d.tobytes(), i.tobytes()))
        e.set_ip_kernel_type(cb.KernelType.Bitwise)
        results[graphs] = out
    assert results[1][-3] != results[1][-2]  # the two refinement forms rank differently here
    assert results[1] == results[0]
    e.close()


@pytest.mark.parametrize("k", [8, 32])
@pytest.mark.parametrize("lanes", [0, 1, 4, 8])
@pytest.mark.parametrize("sfx", ["", "T", "L"])
@pytest.mark.parametrize("D", [64, 128, 192, 768])
def test_refine_sum_order_kat(cb, D, sfx, lanes, k):
    """The refinement's fp64 sums follow the chunked order (eight partials over 16-dim chunks
    mod 8, fixed combination tree) with every lane layout of the refine kernel: on the order
    fixture, where ascending-order summation gives other sums, seeds (k = 32: every vector)
    and main candidates (k = 8) match the oracle bit for bit."""
    from conftest import order_kat_fixture
    sd, q, _ = order_kat_fixture(D)
    ref = po.OracleIndex(sd, **FORMS[sfx]).search(q, k, 1, vanguard=5, with_details=True)
    e = _engine(cb, sd=sd, nq=1, k=k, nprobe=1, **FORMS[sfx])
    e.set_tuning("refine_lanes", lanes)
    e.reset_buffer(q)
    d, i = e.search(q, k, 1)
    e.check_device()
    assert np.array_equal(e.debug("cand_count", 1).astype(np.uint64), ref["cand_count"])
    assert np.array_equal(i, ref["ids"])
    assert d.tobytes() == ref["dist"].tobytes()
    e.close()
