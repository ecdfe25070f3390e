"""The coraanns_search CLI and its C++ headers (options, vector files, recall@k).

CPU: the header unit checks (tests/cpp/check_bench_headers.cpp) and the CLI's argument
errors, which are raised before any device is touched. GPU: the CLI searches the demo golden
index from .fvecs/.ivecs files and must print the recall of the oracle's own top-k
(apps/search.cpp:207-318 report format).
"""
from __future__ import annotations

import re
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, regen_base

PKG = ROOT / "cgcl-coraanns_b200"
CLI = PKG / "_build" / "coraanns_search"


def _build_cli():
    subprocess.run(["make", "-s", "-C", str(PKG), "apps"], check=True, capture_output=True)
    assert CLI.exists()


def _write_vecs(path, arr):
    arr = np.ascontiguousarray(arr)
    n, d = arr.shape
    rec = np.empty((n, d + 1), dtype=np.uint32)
    rec[:, 0] = d
    rec[:, 1:] = arr.view(np.uint32)
    rec.tofile(path)


def _write_bin(path, arr):
    arr = np.ascontiguousarray(arr)
    with open(path, "wb") as f:
        np.array(arr.shape, np.uint32).tofile(f)
        arr.tofile(f)


def test_bench_headers(tmp_path):
    exe = tmp_path / "check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-fopenmp", "-Wall", "-Wextra", "-Werror",
                    f"-I{PKG / 'include'}", f"-I{ROOT / 'include'}",
                    str(ROOT / "tests" / "cpp" / "check_bench_headers.cpp"), "-o", str(exe)],
                   check=True)
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "all checks passed" in r.stdout


def test_cli_argument_errors(tmp_path):
    _build_cli()
    r = subprocess.run([str(CLI)], capture_output=True, text=True)
    assert r.returncode == 1 and "Usage:" in r.stderr
    r = subprocess.run([str(CLI), "a", "b", "c", "--bogus", "1"], capture_output=True, text=True)
    assert r.returncode == 1 and "Unknown option --bogus" in r.stderr
    r = subprocess.run([str(CLI), "a", "b", "c", "--batch-q", "7"], capture_output=True, text=True)
    assert r.returncode == 1 and "batch-q must be in [1, 6]" in r.stderr
    r = subprocess.run([str(CLI), "a", "b", "c", "--queue-capacity", "1000"],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "power of two" in r.stderr
    r = subprocess.run([str(CLI), "a", "b", "c", "--recall-base"], capture_output=True, text=True)
    assert r.returncode == 1 and "Missing file for --recall-base" in r.stderr
    r = subprocess.run([str(CLI), "a", str(tmp_path / "missing.fvecs"), "c"],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "Cannot open vector file" in r.stderr


def _expected_recall(ids, gt_ids, k, dist_radius=None, base=None, queries=None):
    hits = 0
    for q in range(ids.shape[0]):
        truth = set(int(x) for x in gt_ids[q, :k])
        for i in set(int(x) for x in ids[q, :k]):
            if i in truth:
                hits += 1
            elif base is not None and i < base.shape[0]:
                d = np.sum((queries[q].astype(np.float64) - base[i].astype(np.float64)) ** 2)
                hits += d <= dist_radius[q]
    return hits / (ids.shape[0] * k)


def _final_table(stdout):
    lines = stdout.strip().splitlines()
    start = lines.index("nprobe\tQPS\trecall")
    rows = {}
    for line in lines[start + 1:]:
        npb, qps, rec = line.split("\t")
        rows[int(npb)] = (float(qps), float(rec))
    return rows


@pytest.mark.gpu
def test_cli_search_matches_oracle_recall(tmp_path):
    _build_cli()
    z = np.load(GOLDEN / "demo.npz")
    q, gt = z["queries"], z["gt_ids"]
    _write_vecs(tmp_path / "q.fvecs", q)
    _write_vecs(tmp_path / "gt.ivecs", gt)
    cmd = [str(CLI), str(GOLDEN / "demo.index"), str(tmp_path / "q.fvecs"), str(tmp_path / "gt.ivecs"),
           "--topk", "10", "--nprobes", "8,4", "--rounds", "2", "--warmup", "1", "--query-chunk", "37"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    rows = _final_table(r.stdout)
    for npb in (4, 8):
        want = _expected_recall(z[f"ids_k10_np{npb}_v5"], gt, 10)
        assert rows[npb][1] == pytest.approx(want, abs=1e-6)
        assert rows[npb][0] > 0
    assert len(re.findall(r"^\[Run\] round=\d nprobe=\d+ QPS=\S+ recall=", r.stdout, re.M)) == 4

    # distance-aware recall with a .fbin base and --recall-once
    base = regen_base(z["meta"], z["gen"])
    _write_bin(tmp_path / "base.fbin", base)
    radius = np.sum((q.astype(np.float64) - base[gt[:, 9]].astype(np.float64)) ** 2, axis=1)
    cmd = [str(CLI), str(GOLDEN / "demo.index"), str(tmp_path / "q.fvecs"), str(tmp_path / "gt.ivecs"),
           "--topk", "10", "--nprobes", "4", "--rounds", "1", "--warmup", "0",
           "--recall-base", str(tmp_path / "base.fbin"), "--recall-once", "true"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "mode=distance-aware" in r.stdout and "recall=deferred" in r.stdout
    want = _expected_recall(z["ids_k10_np4_v5"], gt, 10, radius, base, q)
    assert _final_table(r.stdout)[4][1] == pytest.approx(want, abs=1e-6)

    # --exact-base: FP32 diagnostic refine; the ids are the oracle's exact-refine ids
    import py_oracle as po
    o = po.oracle_from_file(GOLDEN / "demo.index")
    o.set_exact_base(base)
    _, ids_exact = o.search(q, 10, 4)
    cmd = [str(CLI), str(GOLDEN / "demo.index"), str(tmp_path / "q.fvecs"), str(tmp_path / "gt.ivecs"),
           "--topk", "10", "--nprobes", "4", "--rounds", "1", "--warmup", "0",
           "--exact-base", str(tmp_path / "base.fbin")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "Exact FP32 refine enabled with mmap base:" in r.stdout
    assert _final_table(r.stdout)[4][1] == pytest.approx(_expected_recall(ids_exact, gt, 10),
                                                         abs=1e-6)
    # a base of another shape is rejected before searching
    _write_bin(tmp_path / "short.fbin", base[:100])
    cmd[-1] = str(tmp_path / "short.fbin")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "Exact-refine base shape mismatch" in r.stderr
