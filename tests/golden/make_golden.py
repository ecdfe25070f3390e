#!/usr/bin/env python3
"""Regenerate the committed golden fixtures under tests/golden/.

Runs only where the reference tree was present at build time (it needs
oracle/_ref/libcora_ref_*.so, i.e. the reference's own CPU code). For each fixture it:

1. generates seeded synthetic data (BASELINE config shapes: Gaussian mixtures);
2. trains the IVF partition with a few Lloyd iterations started at the generating centres
   (Faiss is not available; tools/data/train_ivf.py of the reference does k-means + nearest
   assignment);
3. builds the index with the REFERENCE builder (rabitqlib::ivf::IVF::construct + save) and
   stores the index file as written;
4. records the reference's own outputs that pin the oracle: sha256 of every array of the
   reference SearchData adapter, its 7-bit ex-code inner products (ip64_fxu7_avx) on sampled
   (query, vector) pairs, and the reference CPU search (rabitq_cpu loop) result ids;
5. records exact ground truth (fp64, ties by id) and the oracle's search outputs for a grid
   of (topk, nprobe, vanguard), in the default refinement form (the reference's
   128 * ip1 + ip2: keys dist_/ids_/cand_/t1_/probe_/probeg_) and in the full-code form
   (keys with a "T" suffix on the prefix: distT_/idsT_/candT_/t1T_), and with the fp16-LUT
   estimator (the reference's default kernel type; "L" suffix: distL_/idsL_/candL_/t1L_).

Usage: python tests/golden/make_golden.py [names]   (writes tests/golden/*.index, *.npz)
       python tests/golden/make_golden.py --outputs-only [names]
           recomputes step 5 only, from the committed index files (the reference builder
           draws a fresh random rotation on every run, so rebuilding changes the indexes)
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "oracle"))
import py_oracle as po  # noqa: E402

FIXTURES = {
    # name: (n, dim, nlist, nq, sigma, query_noise, seed, grid[, metric]); metric 1 = inner
    # product on unit-normalised vectors
    "demo": (4096, 128, 16, 100, 0.3, 0.05, 20261201,
             [(10, 4, 5), (10, 8, 5), (10, 16, 5), (10, 16, 0), (1, 4, 5), (50, 8, 2)]),
    "d96": (2048, 96, 16, 48, 0.25, 0.05, 20261202,
            [(10, 2, 5), (10, 6, 5), (10, 16, 1), (100, 8, 5), (10, 4, 0)]),
    "d200": (512, 200, 8, 24, 0.3, 0.05, 20261203, [(10, 3, 5), (10, 8, 2), (5, 8, 0)]),
    "d150": (512, 150, 8, 24, 0.3, 0.05, 20261204, [(10, 3, 5), (20, 8, 1)]),
    "ip128": (4096, 128, 16, 64, 0.3, 0.05, 20261207, [(10, 4, 5), (10, 8, 5), (20, 6, 2)], 1),
}


def fixture_metric(name) -> int:
    spec = FIXTURES[name]
    return spec[8] if len(spec) > 8 else 0


def make_data(n, dim, nlist, nq, sigma, qnoise, seed, normalise=False):
    rng = np.random.default_rng(seed)
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    lab = rng.integers(0, nlist, n)
    base = (centres[lab] + sigma * rng.normal(size=(n, dim))).astype(np.float32)
    qlab = rng.integers(0, nlist, nq)
    queries = (centres[qlab] + sigma * rng.normal(size=(nq, dim)) +
               qnoise * rng.normal(size=(nq, dim))).astype(np.float32)
    if normalise:  # unit vectors (the inner-product configurations)
        base = (base / np.linalg.norm(base, axis=1, keepdims=True)).astype(np.float32)
        queries = (queries / np.linalg.norm(queries, axis=1, keepdims=True)).astype(np.float32)
    return centres, base, queries


def lloyd(base, init, iters=10):
    c = init.astype(np.float64).copy()
    b = base.astype(np.float64)
    for _ in range(iters):
        d = (b * b).sum(1)[:, None] + (c * c).sum(1)[None, :] - 2 * b @ c.T
        a = d.argmin(1)
        for j in range(len(c)):
            m = a == j
            if m.any():
                c[j] = b[m].mean(0)
    d = (b * b).sum(1)[:, None] + (c * c).sum(1)[None, :] - 2 * b @ c.T
    return c.astype(np.float32), d.argmin(1).astype(np.uint32)


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def oracle_outputs(oracle, queries, grid, out):
    """The oracle's search outputs over the grid, in both refinement forms, into `out`."""
    for full_code, lut, sfx in ((False, False, ""), (True, False, "T"), (False, True, "L")):
        oracle.full_code, oracle.lut = full_code, lut
        for k, nprobe, van in grid:
            k, nprobe, van = int(k), int(nprobe), int(van)
            det = oracle.search(queries, k, nprobe, vanguard=van, with_details=True)
            tag = f"k{k}_np{nprobe}_v{van}"
            out[f"dist{sfx}_{tag}"] = det["dist"]
            out[f"ids{sfx}_{tag}"] = det["ids"]
            out[f"cand{sfx}_{tag}"] = det["cand_count"]
            out[f"t1{sfx}_{tag}"] = det["thresholds1"]
            if not sfx:
                out[f"probe_{tag}"] = det["probe_ids"]
                out[f"probeg_{tag}"] = det["probe_g"]
    oracle.full_code, oracle.lut = False, False


def refresh_outputs(name):
    """Recompute the oracle outputs of a committed fixture in place (index unchanged)."""
    with np.load(HERE / f"{name}.npz") as z:
        out = {k: z[k] for k in z.files}
    oracle = po.oracle_from_file(HERE / f"{name}.index")
    oracle_outputs(oracle, out["queries"], out["grid"], out)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: outputs refreshed")


def build_fixture(name):
    n, dim, nlist, nq, sigma, qnoise, seed, grid = FIXTURES[name][:8]
    metric = fixture_metric(name)
    centres, base, queries = make_data(n, dim, nlist, nq, sigma, qnoise, seed, metric == 1)
    cents, assign = lloyd(base, centres)
    index_path = HERE / f"{name}.index"
    po.ref_build_index(index_path, base, cents, assign, total_bits=8, metric_ip=metric == 1)
    ref = po.RefIVF(index_path)
    rsd = ref.search_data()
    sd = po.search_data(po.read_ivf_file(index_path))
    for key in ("centroids", "rotator", "short_data", "short_factors", "long_codes", "ex_factors",
                "ids", "sizes"):
        assert np.asarray(sd[key]).tobytes() == np.asarray(rsd[key]).tobytes(), key
    oracle = po.OracleIndex(sd)
    out = {"queries": queries, "gt_ids": None}
    gt_ids, gt_d = po.exact_knn(base, queries, 100, metric)
    out["gt_ids"], out["gt_dist"] = gt_ids, gt_d
    # reference adapter hashes (L0)
    out["sd_sha"] = np.array([sha(rsd[k]) for k in ("centroids", "rotator", "short_data",
                                                    "short_factors", "long_codes", "ex_factors",
                                                    "ids", "sizes")])
    # reference 7-bit ex-code inner products (pins the decoder)
    rng = np.random.default_rng(seed + 7)
    qr = oracle.rotate(queries)
    D = sd["D"]
    lc = D * 7 // 8
    codes = sd["long_codes"].reshape(-1, lc)
    pairs = np.stack([rng.integers(0, nq, 64), rng.integers(0, n, 64)], 1)
    out["ex_pairs"] = pairs.astype(np.int64)
    out["ex_ref_ip"] = np.array([po.ref().ref_ip_ex(qr[a].copy(), codes[b].copy(), D, 7)
                                 for a, b in pairs], np.float32)
    # reference CPU search (rabitq_cpu loop, hacc) for recall-level comparison
    for k, nprobe, _ in grid:
        key = f"refcpu_k{k}_np{nprobe}"
        if key not in out:
            out[key] = ref.search(queries, k, nprobe, threads=4)
    oracle_outputs(oracle, queries, grid, out)
    prep = oracle.query_prep(qr)
    out["qr"] = qr
    out["planes"] = prep["planes"]
    out["scalars"] = np.stack([prep["width"], prep["k1"], prep["kb"], prep["sumq"]], 1)
    out["grid"] = np.array(grid, np.int64)
    out["meta"] = np.array([n, dim, nlist, nq, seed], np.int64)
    out["gen"] = np.array([sigma, qnoise, float(metric == 1)], np.float64)
    out["metric"] = np.array(metric, np.int64)
    ref.close()
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: index {index_path.stat().st_size} B, npz {(HERE / (name + '.npz')).stat().st_size} B")


def main():
    args = sys.argv[1:]
    if args and args[0] == "--outputs-only":
        for name in (args[1:] or FIXTURES):
            refresh_outputs(name)
        return
    if not po.ref_available():
        sys.exit("oracle/_ref is missing: build it with `make -C oracle ref` where the "
                 "reference tree exists")
    for name in (args or FIXTURES):
        build_fixture(name)


if __name__ == "__main__":
    main()
