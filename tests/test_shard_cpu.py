"""Cluster-sharded search, host side, on CPU: world_size-2 gloo ranks.

Each rank holds one shard of a golden index (coraanns_b200.shard.shard_plan /
shard_search_data) behind the oracle's shard backend, and the product's orchestration
(run_sharded_search) exchanges through gloo all-gathers. The merged result must equal the
unsharded oracle's committed result bit for bit: this pins the exchange design (global
threshold from every shard's k smallest seeds, then the top-k of every shard's top-k) that
the CUDA engine implements. Also: every rank derives the same plan, the shards partition the
index, and an inconsistent shard configuration is detected on every rank.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import GOLDEN

CASES = {  # fixture -> (k, nprobe, vanguard) grid points with committed oracle outputs
    "demo": [(10, 4, 5), (10, 8, 5), (10, 16, 0), (1, 4, 5), (50, 8, 2)],
    "d96": [(10, 6, 5), (100, 8, 5), (10, 4, 0)],
    "d200": [(10, 8, 2)],
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, out_q, bad_manifest):
    import sys
    sys.path[:0] = [str(GOLDEN.parent.parent / "oracle"), str(GOLDEN.parent.parent / "cgcl-coraanns_b200")]
    import torch
    import torch.distributed as dist
    import py_oracle as po
    from coraanns_b200 import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        sd = po.search_data(po.read_ivf_file(GOLDEN / f"{name}.index"))
        owner = shard.shard_plan(sd["sizes"], world)
        plans = [torch.zeros(len(owner), dtype=torch.int64) for _ in range(world)]
        dist.all_gather(plans, torch.from_numpy(owner.astype(np.int64)))
        same_plan = all(bool((p.numpy() == owner).all()) for p in plans)
        sub = shard.shard_search_data(sd, owner, rank)
        row = torch.tensor([rank, world + (1 if bad_manifest and rank == 1 else 0), sd["nlist"],
                            sd["dim"], sd["D"], int((owner == rank).sum())], dtype=torch.int64)
        rows = torch.zeros(world * 6, dtype=torch.int64)
        dist.all_gather_into_tensor(rows, row)
        why = shard.manifest_mismatch(rows.numpy().reshape(world, 6))
        results = {}
        if not bad_manifest:
            z = np.load(GOLDEN / f"{name}.npz")
            q = z["queries"]
            exchange = lambda send, recv: dist.all_gather_into_tensor(recv, send)  # noqa: E731
            for k, nprobe, van in CASES[name]:
                backend = po.OracleShard(sub, world, vanguard=van, threads=2)
                out_d = np.empty((len(q), k), np.float32)
                out_i = np.empty((len(q), k), np.uint32)
                shard.run_sharded_search(backend, exchange, q, len(q), k, nprobe, out_d, out_i)
                results[(k, nprobe, van)] = (out_d, out_i, backend.T1)
        out_q.put((rank, same_plan, why, sub["ids"], sub["sizes"], results))
    finally:
        dist.destroy_process_group()


def _run(name, bad_manifest=False, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, q, bad_manifest))
             for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get() for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


@pytest.mark.parametrize("name", sorted(CASES))
def test_sharded_oracle_search_equals_unsharded(name):
    z = np.load(GOLDEN / f"{name}.npz")
    outs = _run(name)
    # every rank derived the same plan; the shards partition the index, order kept
    assert all(o[1] for o in outs)
    assert all(o[2] is None for o in outs)
    import py_oracle as po
    full = po.search_data(po.read_ivf_file(GOLDEN / f"{name}.index"))
    ids = np.concatenate([o[3] for o in outs])
    assert sorted(ids.tolist()) == sorted(full["ids"].tolist())
    sizes = np.stack([o[4].astype(np.int64) for o in outs])
    assert np.array_equal(sizes.sum(0), full["sizes"].astype(np.int64))
    assert ((sizes > 0).sum(0) == (full["sizes"] > 0)).all()  # each cluster on one shard
    for (k, nprobe, van) in CASES[name]:
        want_d, want_i = z[f"dist_k{k}_np{nprobe}_v{van}"], z[f"ids_k{k}_np{nprobe}_v{van}"]
        want_t1 = z[f"t1_k{k}_np{nprobe}_v{van}"]
        for rank, *_rest, res in outs:
            d, i, t1 = res[(k, nprobe, van)]
            assert np.array_equal(i, want_i), (name, k, nprobe, van, rank)
            assert d.tobytes() == want_d.tobytes()
            assert t1.tobytes() == want_t1.tobytes()


def test_inconsistent_shards_are_detected_on_every_rank():
    outs = _run("demo", bad_manifest=True)
    assert all(o[2] is not None and "world sizes differ" in o[2] for o in outs)


def test_manifest_checks():
    from coraanns_b200.shard import manifest_mismatch
    good = [[0, 2, 16, 128, 128, 9], [1, 2, 16, 128, 128, 7]]
    assert manifest_mismatch(good) is None
    assert "ranks" in manifest_mismatch([[0, 2, 16, 128, 128, 9], [0, 2, 16, 128, 128, 7]])
    assert "nlist" in manifest_mismatch([[0, 2, 16, 128, 128, 9], [1, 2, 32, 128, 128, 7]])
    assert "clusters" in manifest_mismatch([[0, 2, 16, 128, 128, 9], [1, 2, 16, 128, 128, 9]])


def test_plan_balances_and_is_deterministic():
    from coraanns_b200.shard import shard_plan
    rng = np.random.default_rng(3)
    sizes = rng.zipf(1.5, 4096).clip(1, 50000).astype(np.uint64)
    for world in (2, 4, 8):
        a, b = shard_plan(sizes, world), shard_plan(sizes.copy(), world)
        assert np.array_equal(a, b)
        load = np.bincount(a, weights=sizes.astype(np.float64), minlength=world)
        # LPT: the most loaded shard exceeds the least by at most one cluster
        assert load.max() - load.min() <= float(sizes.max())
        assert set(np.unique(a)) == set(range(world))
    with pytest.raises(ValueError):
        shard_plan(sizes, 0)


def test_index_file_shard_info_partitions_the_file():
    """A shard engine reads only its clusters' payload from an index file: the shards'
    shares partition the vectors, clusters and payload bytes (no GPU needed)."""
    import coraanns_b200 as cb
    import py_oracle as po
    path = GOLDEN / "d96.index"
    whole = cb.index_file_shard_info(path, 0, 1)
    ivf = po.read_ivf_file(path)
    assert whole["vectors"] == whole["total_vectors"] == int(ivf["num"])
    assert whole["clusters"] == int(ivf["nlist"])
    for world in (2, 3, 4):
        parts = [cb.index_file_shard_info(path, r, world) for r in range(world)]
        assert sum(p["vectors"] for p in parts) == whole["vectors"]
        assert sum(p["clusters"] for p in parts) == whole["clusters"]
        assert sum(p["payload_bytes"] for p in parts) == whole["payload_bytes"]
        assert max(p["payload_bytes"] for p in parts) < whole["payload_bytes"]


def test_index_file_shard_info_rejects_bad_arguments(tmp_path):
    import coraanns_b200 as cb
    path = GOLDEN / "d96.index"
    for rank, world in ((2, 2), (0, 0), (0, 1000)):
        with pytest.raises(ValueError):
            cb.index_file_shard_info(path, rank, world)
    with pytest.raises(ValueError):
        cb.index_file_shard_info(tmp_path / "missing.index", 0, 1)
