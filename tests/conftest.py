"""Shared test setup: the gpu marker, import paths, golden fixtures and KAT builders."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "cgcl-coraanns_b200"))
sys.path.insert(0, str(ROOT))

GOLDEN_NAMES = ["demo", "d96", "d200", "d150", "ip128"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def golden():
    """name -> (index path, npz dict)."""
    out = {}
    for name in GOLDEN_NAMES:
        with np.load(GOLDEN / f"{name}.npz") as z:
            out[name] = (GOLDEN / f"{name}.index", {k: z[k] for k in z.files})
    return out


def regen_base(meta, gen):
    """Regenerate a fixture's base vectors from its recorded seed (make_golden.make_data);
    gen[2], when present, marks unit-normalised (inner-product) fixtures."""
    n, dim, nlist, nq, seed = (int(x) for x in meta)
    sigma = float(gen[0])
    rng = np.random.default_rng(seed)
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    lab = rng.integers(0, nlist, n)
    base = (centres[lab] + sigma * rng.normal(size=(n, dim))).astype(np.float32)
    if len(gen) > 2 and gen[2]:
        base = (base / np.linalg.norm(base, axis=1, keepdims=True)).astype(np.float32)
    return base


def fixture_metric(z) -> int:
    """0 squared L2, 1 inner product (fixtures record it; older ones are L2)."""
    return int(z["metric"]) if "metric" in z else 0


# ------------------------------------------------------------------------------------
# Known-answer fixtures ported from the reference's GPU tests
# (tests/gpu_cpu_ring_queue_test.cpp:17-50, tests/gpu_cpu_highk_vanguard_test.cpp:82-107,
#  tests/gpu_search_lifecycle_test.cpp:18-37): identity rotation, all-zero codes,
# f_add = -1e6 so that every vector passes the 1-bit filter, unique f_add_ex.
# ------------------------------------------------------------------------------------
def kat_fixture(count=32768, topk=100, clusters=8, queries=5, dim=96, padded=128, f_add=-1e6):
    sd = dict(num=count, dim=dim, D=padded, nlist=clusters, ex_bits=7)
    sd["centroids"] = np.zeros((clusters, padded), np.float32)
    rot = np.zeros((dim, padded), np.float32)
    rot[np.arange(dim), np.arange(dim)] = 1.0
    sd["rotator"] = rot
    sd["short_data"] = np.zeros(count * padded // 32, np.uint32)
    sf = np.zeros((count, 3), np.float32)
    sf[:, 0] = f_add
    sd["short_factors"] = sf
    sd["long_codes"] = np.zeros(count * padded * 7 // 8, np.uint8)
    lf = np.zeros((count, 2), np.float32)
    i = np.arange(count, dtype=np.int64)
    lf[:, 0] = (0.01 * ((i * 7919) % count).astype(np.float32)).astype(np.float32)
    sd["ex_factors"] = lf
    sd["ids"] = np.arange(count, dtype=np.uint32)
    sd["sizes"] = np.full(clusters, count // clusters, np.uint64)
    q = np.zeros((queries, dim), np.float32)
    for a in range(queries):
        for d in range(dim):
            q[a, d] = np.float32(0.01) * np.float32(1 + (a + d) % 7)
    order = np.argsort(lf[:, 0], kind="stable")
    expected = np.sort(order[:topk]).astype(np.uint32)
    return sd, q, expected


# ------------------------------------------------------------------------------------
# Summation-order known-answer fixture of the refinement's fp64 inner product: identity
# rotation, one cluster whose centroid is the query (g = 0), all-zero 1-bit codes and scan
# factors (ip1 = 0, every low 0), ex factors (0, 1), so each vector's distance is
# ip2 + kb with ip2 = <q, u>. The query puts +-2^55 at the first dimension of every 16-dim
# chunk (alternating sign), 1 at the second and a small value at the third; each vector has
# u = 1 at dims 16a, 16a + 1, 16b, 16b + 1 (chunks a < b of opposite sign) and small codes at
# every third dimension. In ascending dimension order every term between the two large ones
# is rounded against 2^55; in the chunked order (partial sums over chunks mod 8) the large
# terms sit in their own partials, so the two orders give different sums.
# ------------------------------------------------------------------------------------
def order_kat_fixture(D, n=32):
    import torch
    from coraanns_b200 import builder
    nch = D // 16
    q = np.zeros(D, np.float32)
    for k in range(nch):
        q[16 * k] = np.float32((1 if k % 2 == 0 else -1) * 2.0 ** 55)
        q[16 * k + 1] = 1.0
        q[16 * k + 2] = np.float32(0.125 * (k + 1))
    rng = np.random.default_rng(D)
    u = np.zeros((n, D), np.uint8)
    for v in range(n):
        a = int(rng.integers(0, nch - 1))
        b = int(rng.integers(a + 1, nch))
        if (b - a) % 2 == 0:  # b > a + 1 here: b - 1 keeps a < b and flips the sign
            b -= 1
        for c in (a, b):
            u[v, 16 * c] = 1
            u[v, 16 * c + 1] = 1
        for k in range(nch):
            u[v, 16 * k + 2] = (v + 3 * k) % 128
    sd = dict(num=n, dim=D, D=D, nlist=1, ex_bits=7)
    sd["centroids"] = q[None, :].copy()
    sd["rotator"] = np.eye(D, dtype=np.float32)
    sd["short_data"] = np.zeros(n * D // 32, np.uint32)
    sd["short_factors"] = np.zeros((n, 3), np.float32)
    sd["long_codes"] = builder._pack_ex7(torch.from_numpy(u)).numpy().reshape(-1)
    ef = np.zeros((n, 2), np.float32)
    ef[:, 1] = 1.0
    sd["ex_factors"] = ef
    sd["ids"] = np.arange(n, dtype=np.uint32)
    sd["sizes"] = np.array([n], np.uint64)
    return sd, q[None, :].copy(), u
