"""CPU tests: the oracle pinned against the reference's own outputs and known answers.

These never touch a GPU. They establish that oracle/cora_oracle.c restates the reference
path faithfully before any CUDA result is compared against it.
"""
from __future__ import annotations

import ctypes as C
import hashlib

import numpy as np
import pytest

import py_oracle as po
from conftest import GOLDEN_NAMES, fixture_metric, kat_fixture, regen_base

SD_KEYS = ("centroids", "rotator", "short_data", "short_factors", "long_codes", "ex_factors",
           "ids", "sizes")


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_searchdata_restatement_matches_reference_hashes(golden, name):
    """L0 layout: the numpy restatement of src/index/search_data.cpp:45-123 reproduces the
    reference adapter's arrays byte for byte (hashes recorded from the compiled reference)."""
    path, z = golden[name]
    sd = po.search_data(po.read_ivf_file(path))
    got = [hashlib.sha256(np.ascontiguousarray(sd[k]).tobytes()).hexdigest() for k in SD_KEYS]
    assert got == list(z["sd_sha"])


MODES = {"": dict(), "T": dict(full_code=True), "L": dict(lut=True)}


@pytest.mark.parametrize("sfx", list(MODES))
@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_oracle_reproduces_golden_outputs(golden, name, sfx):
    """The oracle is deterministic: rerunning it gives the committed outputs bit for bit, with
    the integer estimator and the reference's refinement (the default), the full-code
    refinement ("T" keys) and the fp16-LUT estimator ("L" keys)."""
    path, z = golden[name]
    o = po.oracle_from_file(path, **MODES[sfx])
    for k, nprobe, van in z["grid"]:
        tag = f"k{k}_np{nprobe}_v{van}"
        det = o.search(z["queries"], int(k), int(nprobe), vanguard=int(van), with_details=True)
        assert np.array_equal(det["ids"], z[f"ids{sfx}_{tag}"]), tag
        assert det["dist"].tobytes() == z[f"dist{sfx}_{tag}"].tobytes(), tag
        assert np.array_equal(det["cand_count"], z[f"cand{sfx}_{tag}"]), tag
        assert det["thresholds1"].tobytes() == z[f"t1{sfx}_{tag}"].tobytes(), tag
        assert np.array_equal(det["probe_ids"], z[f"probe_{tag}"]), tag


def _pair_terms(sd, z, o):
    """Per recorded (query, vector) pair: the oracle's ip1 (width * ip_int), the vector's
    coarse distance g to its own cluster's centroid, the query's kb, and the ex factors."""
    D = int(sd["D"])
    starts = np.concatenate([[0], np.cumsum(sd["sizes"].astype(np.int64))])
    prep = o.query_prep(z["qr"])
    out = []
    for qi, gid in z["ex_pairs"]:
        qi, gid = int(qi), int(gid)
        c = int(np.searchsorted(starts, gid, side="right") - 1)
        ip_int = po.lib().cora_oracle_ip_int(C.byref(o.c), gid,
                                             np.ascontiguousarray(prep["planes"][qi]))
        ip1 = np.float32(prep["width"][qi]) * np.float32(ip_int)
        x = np.ascontiguousarray(z["qr"][qi])
        out.append((qi, gid, np.float32(ip1), _g_add(sd, x, c), np.float32(prep["kb"][qi])))
    return out


def _g_add(sd, x, c):
    """The additive query term of cluster c: the squared distance (L2) or -<q', c'> (IP)."""
    cent = np.ascontiguousarray(sd["centroids"][c])
    D = int(sd["D"])
    if int(sd.get("metric", 0)) == 1:
        return np.float32(po.lib().cora_oracle_ip_gadd(x, cent, D))
    return np.float32(po.lib().cora_oracle_centroid_dist(x, cent, D))


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_ex_code_inner_product_matches_reference_decoder(golden, name):
    """ip2 = <q', u> of the oracle (fp64, rounded once) equals the reference's ip64_fxu7_avx
    (third_party/.../utils/space.hpp:677-762, fp32 AVX sums, recorded) on sampled pairs
    within 1e-4 relative."""
    path, z = golden[name]
    sd = po.search_data(po.read_ivf_file(path))
    D = int(sd["D"])
    codes = sd["long_codes"].reshape(-1, D * 7 // 8)
    for (qi, gid), ref_ip in zip(z["ex_pairs"], z["ex_ref_ip"]):
        mine = po.lib().cora_oracle_ip_ex(np.ascontiguousarray(z["qr"][qi]),
                                          codes[gid].copy(), D)
        assert abs(mine - float(ref_ip)) <= 1e-4 * max(1.0, abs(float(ref_ip))), (qi, gid)


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_refinement_matches_reference_expression(golden, name):
    """The default refinement is the reference's: the reference's own expression
    f_add_ex + g + f_rescale_ex * ((2^7 * exact_ip + ip2) + kb) (cpu_refinement.cpp:186-191),
    evaluated here in fp32 with the reference's ip2 (ip64_fxu7_avx, recorded) and the scan's
    exact_ip (width * ip_int, filter_kernels.cuh:106), agrees with the oracle's distance
    within 1e-4 relative (of the distance's magnitude, floored at 1) on every sampled pair."""
    path, z = golden[name]
    sd = po.search_data(po.read_ivf_file(path))
    o = po.OracleIndex(sd)
    D = int(sd["D"])
    codes = sd["long_codes"].reshape(-1, D * 7 // 8)
    f32 = np.float32
    worst = 0.0
    for (qi, gid, ip1, g, kb), ref_ip2 in zip(_pair_terms(sd, z, o), z["ex_ref_ip"]):
        fa, fr = (f32(v) for v in sd["ex_factors"][gid])
        ref_ex = (fa + g) + fr * ((f32(128) * ip1 + f32(ref_ip2)) + kb)
        ip2 = po.lib().cora_oracle_ip_ex(np.ascontiguousarray(z["qr"][qi]), codes[gid].copy(), D)
        mine = po.lib().cora_oracle_ex_split(C.byref(o.c), gid, float(ip1), ip2, float(g),
                                             float(kb))
        err = abs(mine - float(ref_ex)) / max(1.0, abs(float(ref_ex)))
        worst = max(worst, err)
    assert worst <= 1e-4, worst


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")
@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_refinement_matches_reference_expression_live(golden, name):
    """As above with the reference's ip64_fxu7_avx run live, on every candidate the oracle
    refines for the first queries (seeds and main candidates of one grid point)."""
    path, z = golden[name]
    sd = po.search_data(po.read_ivf_file(path))
    o = po.OracleIndex(sd)
    D = int(sd["D"])
    codes = sd["long_codes"].reshape(-1, D * 7 // 8)
    k, nprobe, van = (int(v) for v in z["grid"][0])
    q = z["queries"][:6]
    det = o.search(q, k, nprobe, vanguard=van, with_details=True, cand_cap=4096)
    prep = o.query_prep(z["qr"][:6])
    starts = np.concatenate([[0], np.cumsum(sd["sizes"].astype(np.int64))])
    f32 = np.float32
    worst, count = 0.0, 0
    for qi in range(len(q)):
        x = np.ascontiguousarray(z["qr"][qi])
        for gid in det["cand_gids"][qi]:
            if gid == 0xFFFFFFFF:
                break
            gid = int(gid)
            c = int(np.searchsorted(starts, gid, side="right") - 1)
            g = _g_add(sd, x, c)
            ip_int = po.lib().cora_oracle_ip_int(C.byref(o.c), gid,
                                                 np.ascontiguousarray(prep["planes"][qi]))
            ip1 = f32(prep["width"][qi]) * f32(ip_int)
            kb = f32(prep["kb"][qi])
            ref_ip2 = f32(po.ref().ref_ip_ex(x, codes[gid].copy(), D, 7))
            fa, fr = (f32(v) for v in sd["ex_factors"][gid])
            ref_ex = (fa + g) + fr * ((f32(128) * ip1 + ref_ip2) + kb)
            ip2 = po.lib().cora_oracle_ip_ex(x, codes[gid].copy(), D)
            mine = po.lib().cora_oracle_ex_split(C.byref(o.c), gid, float(ip1), ip2, float(g),
                                                 float(kb))
            worst = max(worst, abs(mine - float(ref_ex)) / max(1.0, abs(float(ref_ex))))
            count += 1
    assert count > 0 and worst <= 1e-4, (count, worst)


def test_half_conversion_matches_ieee_round_to_nearest_even():
    """The oracle's binary32 -> binary16 rounding (the LUT entries; CUDA's __float2half_rn)
    equals numpy's IEEE conversion on random values across the half range, subnormals, ties
    and overflow; binary16 -> binary32 is exact for every finite half."""
    rng = np.random.default_rng(5)
    v = (rng.normal(size=50000) * 10.0 ** rng.integers(-9, 6, 50000)).astype(np.float32)
    edges = np.array([0.0, -0.0, 65504, 65519.996, 65520, -65520, 1e9, 2 ** -24, 2 ** -25,
                      3 * 2 ** -26, 2 ** -14, 2 ** -14 * (1 - 2 ** -11), 1 + 2 ** -11,
                      1 + 3 * 2 ** -11], np.float32)
    v = np.concatenate([v, edges])
    with np.errstate(over="ignore"):
        want = v.astype(np.float16).view(np.uint16)
    got = np.array([po.lib().cora_oracle_f32_to_f16(float(x)) for x in v], np.uint16)
    assert np.array_equal(got, want)
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    back = np.array([po.lib().cora_oracle_f16_to_f32(int(x)) for x in h], np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(back[fin].view(np.uint32), ref[fin].view(np.uint32))


def test_lut_tables_restate_reference_formula(golden):
    """query_kernels.cuh:199-221: entry (g, p) = half(fp32 sum from 0 of the q'[4g + i]
    selected by bit 3 - i of p, i ascending), restated here in numpy and compared bitwise."""
    path, z = golden["d96"]
    o = po.oracle_from_file(path)
    qr = z["qr"][:8]
    got = o.query_lut(qr)
    D = qr.shape[1]
    want = np.zeros((len(qr), D // 4, 16), np.float16)
    for p in range(16):
        acc = np.zeros((len(qr), D // 4), np.float32)
        for i in range(4):
            if p & (8 >> i):
                acc = (acc + qr[:, i::4]).astype(np.float32)
        want[:, :, p] = acc.astype(np.float16)
    assert np.array_equal(got, want.view(np.uint16))


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_recall_on_par_with_reference_cpu(golden, name):
    """L5: distance-aware recall@k against the reference CPU search (the rabitq_cpu loop,
    recorded). The fp16-LUT estimator (the reference hybrid path's default kernel type) and
    the full-code refinement are at least the reference's minus 0.02 at every grid point. The
    default form reproduces the reference hybrid path's 128 * ip1 + ip2 with the integer
    estimator's ip1 (its Bitwise kernel type), whose 8-bit query quantisation costs recall
    against rabitq_cpu's estimator: it is held to 0.06 below it."""
    path, z = golden[name]
    base = regen_base(z["meta"], z["gen"])
    gt = z["gt_ids"]
    m = fixture_metric(z)
    assert np.array_equal(po.exact_knn(base, z["queries"][:4], 10, m)[0], gt[:4, :10])
    for k, nprobe, van in z["grid"]:
        tag = f"k{k}_np{nprobe}_v{van}"
        ref = po.distance_recall(base, z["queries"], gt, z[f"refcpu_k{k}_np{nprobe}"], int(k), m)
        for sfx in ("T", "L"):
            other = po.distance_recall(base, z["queries"], gt, z[f"ids{sfx}_{tag}"], int(k), m)
            assert other >= ref - 0.02, (tag, sfx, other, ref)
        if int(k) >= 10:
            mine = po.distance_recall(base, z["queries"], gt, z[f"ids_{tag}"], int(k), m)
            assert mine >= ref - 0.06, (tag, mine, ref)


def test_inner_product_fixture_is_searched_as_inner_product(golden):
    """The IP fixture's header says METRIC_IP; the oracle's results rank by the estimate of
    1 - <q, x>: its top-1 id has, on most queries, the largest exact inner product."""
    path, z = golden["ip128"]
    assert po.read_ivf_file(path)["metric"] == 1 and fixture_metric(z) == 1
    base = regen_base(z["meta"], z["gen"])
    ids = z["ids_k10_np8_v5"]
    ip = np.einsum("qd,qd->q", base[ids[:, 0]].astype(np.float64), z["queries"].astype(np.float64))
    best = (base.astype(np.float64) @ z["queries"].astype(np.float64).T).max(0)
    assert np.mean(np.isclose(ip, best)) >= 0.9
    d = z["dist_k10_np8_v5"]
    assert np.all(np.abs(d[:, 0] - (1 - best)) < 0.1)


def test_query_prep_matches_reference_formulas(golden):
    """query_kernels.cuh:117-189: planes reconstruct qint exactly; width = amax / 127."""
    _, z = golden["demo"]
    o = po.oracle_from_file(golden["demo"][0])
    prep = o.query_prep(z["qr"])
    qint = prep["qint"]
    assert qint.min() >= -128 and qint.max() <= 127
    amax = np.abs(z["qr"]).max(1)
    assert np.array_equal(prep["width"], np.maximum(amax / np.float32(127), np.float32(1e-30)))
    D = z["qr"].shape[1]
    for q in range(4):
        rec = np.zeros(D, np.int64)
        for b in range(8):
            for j in range(D):
                bit = (prep["planes"][q, b, j // 32] >> (31 - j % 32)) & 1
                rec[j] += int(bit) << b
        rec = np.where(rec >= 128, rec - 256, rec)
        assert np.array_equal(rec, qint[q])
    assert np.array_equal(prep["planes"], z["planes"])


# ------------------------------------------------------------------------------------
# known-answer tests of the reference's GPU suite, run on the oracle
# ------------------------------------------------------------------------------------
@pytest.mark.parametrize("vanguard", [0, 5])
def test_kat_exact_ids_and_payloads(vanguard):
    """gpu_cpu_ring_queue_test.cpp:67-98: every vector is a candidate (count n*N), ids are
    the smallest f_add_ex, distances = f_add_ex + ||q||^2 within 1e-4."""
    sd, q, expected = kat_fixture()
    o = po.OracleIndex(sd)
    det = o.search(q, 100, 8, vanguard=vanguard, with_details=True)
    assert det["cand_count"].tolist() == [32768] * 5
    for a in range(5):
        assert np.array_equal(np.sort(det["ids"][a]), expected)
        qn = np.float32(0)
        for d in range(96):
            qn = np.float32(qn + q[a, d] * q[a, d])
        exp = sd["ex_factors"][det["ids"][a], 0] + qn
        assert np.abs(det["dist"][a] - exp).max() < 1e-4


def test_kat_empty_results_are_flt_max():
    """gpu_cpu_ring_queue_test.cpp:148-167: f_add = FLT_MAX -> no candidates, FLT_MAX out."""
    sd, q, _ = kat_fixture(f_add=np.finfo(np.float32).max)
    det = po.OracleIndex(sd).search(q, 100, 8, with_details=True)
    assert det["cand_count"].sum() == 0
    assert np.all(det["dist"] == np.finfo(np.float32).max) and np.all(det["ids"] == 0)


def test_kat_seeded_negative_thresholds_reject_everything():
    """gpu_cpu_ring_queue_test.cpp:192-199: thresholds seeded to -FLT_MAX -> 0 candidates."""
    sd, q, _ = kat_fixture()
    t = np.full(5, -np.finfo(np.float32).max, np.float32)
    det = po.OracleIndex(sd).search(q, 100, 8, thresholds=t, with_details=True)
    assert det["cand_count"].sum() == 0


@pytest.mark.parametrize("k", [10, 100, 513, 1024])
def test_kat_highk_vanguard_on_off_agree(k):
    """gpu_cpu_highk_vanguard_test.cpp:146-183: vanguard on/off and chunking give identical
    ids and distances; ids are the k smallest f_add_ex."""
    sd, q, _ = kat_fixture(topk=k)
    o = po.OracleIndex(sd)
    d0, i0 = o.search(q, k, 8, vanguard=0)
    d5, i5 = o.search(q, k, 8, vanguard=5)
    d2, i2 = o.search(q[:2], k, 8, vanguard=5)
    assert np.array_equal(i0, i5) and d0.tobytes() == d5.tobytes()
    assert np.array_equal(i2, i5[:2]) and d2.tobytes() == d5[:2].tobytes()
    order = np.argsort(sd["ex_factors"][:, 0], kind="stable")[:k]
    assert np.array_equal(np.sort(i0[0]), np.sort(order.astype(np.uint32)))


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")
def test_searchdata_restatement_matches_live_reference(golden):
    """Same as the hash test, against the compiled reference adapter run live."""
    path, _ = golden["d96"]
    rsd = po.RefIVF(path).search_data()
    sd = po.search_data(po.read_ivf_file(path))
    for k in SD_KEYS:
        assert np.asarray(sd[k]).tobytes() == np.asarray(rsd[k]).tobytes(), k


@pytest.mark.parametrize("D", [64, 128, 192, 768])
def test_refinement_sum_order_kat(D):
    """The oracle's ip2 follows the chunked summation order (eight partial sums over the
    16-dim chunks mod 8, combined ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7))), and on
    the order fixture that order differs from ascending-dimension summation."""
    from conftest import order_kat_fixture
    sd, q, u = order_kat_fixture(D)
    codes = np.asarray(sd["long_codes"]).reshape(sd["num"], D * 7 // 8)
    x = np.ascontiguousarray(q[0])
    differs = 0
    for v in range(sd["num"]):
        mine = po.lib().cora_oracle_ip_ex(x, codes[v].copy(), D)
        terms = x.astype(np.float64) * u[v].astype(np.float64)
        p = [0.0] * 8
        for d in range(D):
            p[(d // 16) % 8] += float(terms[d])
        chunked = np.float32(((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7])))
        seq = 0.0
        for d in range(D):
            seq += float(terms[d])
        assert np.float32(mine).tobytes() == chunked.tobytes()
        differs += np.float32(seq) != chunked
    assert differs >= sd["num"] // 2, differs
