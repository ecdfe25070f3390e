"""Cluster-sharded search on the GPU: the shard kernels and the exchange protocol.

On one GPU, `world` sharded engines of one index run in one process and exchange through
device copies (the all-gather a multi-GPU run does with NCCL): the merged result must equal
the oracle's committed result, and the unsharded engine's, bit for bit. With two or more
GPUs, two torch.distributed ranks over NCCL run the same check through ShardedIndex.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb():
    import coraanns_b200
    return coraanns_b200


class LocalShards:
    """`world` shard engines of one index on this GPU, exchanging by device copies."""

    def __init__(self, cb, load, world, nq, k, nprobe, vanguard=5, lows=True):
        self.engines = []
        for r in range(world):
            e = cb.HybridIndex(0)
            e.shard_configure(r, world)
            e.set_vanguard_size(vanguard)
            if not lows:
                e.set_vanguard_lows_budget(0)
            load(e)
            e.prepare_workspace(nq, k, nprobe)
            self.engines.append(e)

    def search(self, q, k, nprobe, split=False):
        import torch
        from coraanns_b200.shard import exchange_words, probe_words
        nq, world = q.shape[0], len(self.engines)
        w = exchange_words(nq, k)
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
            sends = [torch.empty(w, dtype=torch.int64, device="cuda") for _ in range(world)]
            recv = torch.empty(world * w, dtype=torch.int64, device="cuda")
            outs = [(torch.empty((nq, k), dtype=torch.float32, device="cuda"),
                     torch.empty((nq, k), dtype=torch.int32, device="cuda")) for _ in range(world)]
            if split:  # each engine probes its slice of the queries; the lists are exchanged
                pw = probe_words(nq, nprobe, world)
                psends = [torch.empty(pw, dtype=torch.int64, device="cuda") for _ in range(world)]
                precv = torch.empty(world * pw, dtype=torch.int64, device="cuda")
                for e, ps in zip(self.engines, psends):
                    e.shard_search_probe(dq.data_ptr(), nq, k, nprobe, ps.data_ptr(), st.cuda_stream)
                torch.cat(psends, out=precv)
                for e, s in zip(self.engines, sends):
                    e.shard_search_begin_probed(precv.data_ptr(), s.data_ptr())
            else:
                for e, s in zip(self.engines, sends):
                    e.shard_search_begin(dq.data_ptr(), nq, k, nprobe, s.data_ptr(), st.cuda_stream)
            torch.cat(sends, out=recv)
            for e, s in zip(self.engines, sends):
                e.shard_search_resume(recv.data_ptr(), s.data_ptr())
            torch.cat(sends, out=recv)
            for e, (d, i) in zip(self.engines, outs):
                e.shard_search_end(recv.data_ptr(), d.data_ptr(), i.data_ptr())
        st.synchronize()
        for e in self.engines:
            e.check_device()
        return [(d.cpu().numpy(), i.cpu().numpy().view(np.uint32)) for d, i in outs]

    def close(self):
        for e in self.engines:
            e.close()


CASES = [("demo", 10, 8, 5), ("demo", 50, 8, 2), ("demo", 10, 16, 0), ("d96", 100, 8, 5),
         ("d200", 10, 8, 2), ("d150", 20, 8, 1)]


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("lows", [True, False])
@pytest.mark.parametrize("name,k,nprobe,van", CASES)
def test_local_shards_match_oracle(cb, name, k, nprobe, van, world, lows, split):
    z = np.load(GOLDEN / f"{name}.npz")
    q = z["queries"]
    path = str(GOLDEN / f"{name}.index")
    ls = LocalShards(cb, lambda e: e.load_index_file(path), world, len(q), k, nprobe, van, lows)
    outs = ls.search(q, k, nprobe, split=split)
    want_d, want_i = z[f"dist_k{k}_np{nprobe}_v{van}"], z[f"ids_k{k}_np{nprobe}_v{van}"]
    for d, i in outs:
        assert np.array_equal(i, want_i)
        assert d.tobytes() == want_d.tobytes()
    # every shard applied the global threshold; the shards' candidates add up to the
    # unsharded candidate count (each candidate lives on exactly one shard)
    t1 = [e.debug("thresholds1", len(q)) for e in ls.engines]
    for t in t1:
        assert t.tobytes() == z[f"t1_k{k}_np{nprobe}_v{van}"].tobytes()
    cand = sum(e.debug("cand_count", len(q)).astype(np.int64) for e in ls.engines)
    assert np.array_equal(cand, z[f"cand_k{k}_np{nprobe}_v{van}"].astype(np.int64))
    info = [e.shard_info() for e in ls.engines]
    assert sum(x["clusters"] for x in info) == int(z["meta"][2])
    ls.close()


def test_local_shards_synthetic_match_unsharded(cb):
    """World 4 over a larger index (heavier clusters, several tiles per cluster)."""
    from coraanns_b200 import builder
    rng = np.random.default_rng(17)
    n, dim, nlist, nq, k, nprobe = 200_000, 96, 256, 512, 10, 16
    centres = rng.normal(size=(nlist, dim)).astype(np.float32)
    lab = rng.integers(0, nlist, n)
    data = (centres[lab] + 0.25 * rng.normal(size=(n, dim))).astype(np.float32)
    q = (centres[rng.integers(0, nlist, nq)] + 0.25 * rng.normal(size=(nq, dim))).astype(np.float32)
    sd = builder.build_index(data, centres, lab, seed=17)
    full = cb.HybridIndex(0)
    full.load_search_data(sd)
    full.prepare_workspace(nq, k, nprobe)
    full.reset_buffer(q)
    want_d, want_i = full.search(q, k, nprobe)
    full.close()
    ls = LocalShards(cb, lambda e: e.load_search_data(sd), 4, nq, k, nprobe)
    for split in (False, True):
        for d, i in ls.search(q, k, nprobe, split=split):
            assert np.array_equal(i, want_i) and d.tobytes() == want_d.tobytes()
    ls.close()


def test_shard_arrays_built_per_shard_match_whole_index(cb):
    """Shard engines loaded from arrays of their own clusters only (cora_load_shard_arrays),
    each built alone by per-shard generation, search bit-identically to the engine that
    holds the whole index; a local size that disagrees with the plan is rejected."""
    import torch
    from coraanns_b200 import synthetic
    from coraanns_b200.shard import exchange_words, shard_plan
    mix = synthetic.ComponentShards(400_000, 96, 512, 0.25, seed=3, device="cuda")
    world, k, nprobe = 3, 10, 16
    owner = shard_plan(mix.counts, world)
    q = mix.queries(256, 0.05).cpu().numpy()
    whole = synthetic.build_shard(mix, np.zeros(mix.ncomp, np.int32), 0, seed=5)
    e = cb.HybridIndex(0)
    e.load_search_data(whole)
    e.prepare_workspace(len(q), k, nprobe)
    e.reset_buffer(q)
    want_d, want_i = e.search(q, k, nprobe)
    e.close()
    engines = []
    for r in range(world):
        s = cb.HybridIndex(0)
        s.shard_configure(r, world)
        s.load_shard_arrays(synthetic.build_shard(mix, owner, r, seed=5), mix.counts)
        s.prepare_workspace(len(q), k, nprobe)
        engines.append(s)
    w = exchange_words(len(q), k)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dq = torch.from_numpy(q).cuda()
        sends = [torch.empty(w, dtype=torch.int64, device="cuda") for _ in range(world)]
        recv = torch.empty(world * w, dtype=torch.int64, device="cuda")
        od = torch.empty((len(q), k), dtype=torch.float32, device="cuda")
        oi = torch.empty((len(q), k), dtype=torch.int32, device="cuda")
        for s, b in zip(engines, sends):
            s.shard_search_begin(dq.data_ptr(), len(q), k, nprobe, b.data_ptr(), st.cuda_stream)
        torch.cat(sends, out=recv)
        for s, b in zip(engines, sends):
            s.shard_search_resume(recv.data_ptr(), b.data_ptr())
        torch.cat(sends, out=recv)
        engines[0].shard_search_end(recv.data_ptr(), od.data_ptr(), oi.data_ptr())
    st.synchronize()
    for s in engines:
        s.check_device()
        s.close()
    assert np.array_equal(oi.cpu().numpy().view(np.uint32), want_i)
    assert od.cpu().numpy().tobytes() == want_d.tobytes()
    bad = synthetic.build_shard(mix, owner, 0, seed=5)
    bad["sizes"] = bad["sizes"].copy()
    c = int(np.flatnonzero(owner != 0)[0])
    bad["sizes"][c] = 1
    s = cb.HybridIndex(0)
    s.shard_configure(0, world)
    with pytest.raises(cb.InvalidArgument, match="plan"):
        s.load_shard_arrays(bad, mix.counts)
    s.close()


def test_sharded_engine_rules(cb):
    path = str(GOLDEN / "demo.index")
    e = cb.HybridIndex(0)
    with pytest.raises(cb.InvalidArgument):
        e.shard_configure(2, 2)
    e.shard_configure(1, 2)
    e.load_index_file(path)
    with pytest.raises(cb.LogicError):
        e.shard_configure(0, 2)  # after loading
    e.prepare_workspace(8, 10, 4)
    q = np.load(GOLDEN / "demo.npz")["queries"][:8]
    with pytest.raises(cb.LogicError, match="shard"):
        e.search(q, 10, 4)  # a shard alone cannot answer
    with pytest.raises(cb.LogicError):
        e.shard_search_resume(1, 1)  # before begin
    with pytest.raises(cb.LogicError, match="probe"):
        e.shard_search_begin_probed(1, 1)  # before probe
    info = e.shard_info()
    assert info["rank"] == 1 and info["world"] == 2 and 0 < info["vectors"] < 4096
    e.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_q):
    import sys
    root = GOLDEN.parent.parent
    sys.path[:0] = [str(root / "cgcl-coraanns_b200"), str(root / "tests")]
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from coraanns_b200.shard import ShardedIndex
        z = np.load(GOLDEN / "d96.npz")
        q = z["queries"]
        ix = ShardedIndex(rank)
        ix.load_index_file(str(GOLDEN / "d96.index"))
        ix.prepare_workspace(len(q), 100, 8)
        d, i = ix.search(q, 100, 8)
        ok = np.array_equal(i, z["ids_k100_np8_v5"]) and d.tobytes() == z["dist_k100_np8_v5"].tobytes()
        # the whole sharded search (engine launches + both all-gathers) captured in one CUDA
        # graph and replayed twice returns the same bytes
        dq = torch.from_numpy(q).cuda()
        od = torch.full((len(q), 100), -1.0, device="cuda")
        oi = torch.full((len(q), 100), -1, dtype=torch.int32, device="cuda")
        ix.capture(dq, 100, 8, od, oi)
        for _ in range(2):
            od.fill_(-1.0)
            ix.replay()
            torch.cuda.synchronize()
            ix.engine.check_device()
            ok = ok and np.array_equal(oi.cpu().numpy().view(np.uint32), i) and \
                od.cpu().numpy().tobytes() == d.tobytes()
        # the same search with every shard probing the whole batch (no probe exchange)
        ix.split_probe = False
        d2, i2 = ix.search(q, 100, 8)
        ok = ok and np.array_equal(i2, i) and d2.tobytes() == d.tobytes()
        # and in query chunks (an uneven last chunk), probing split again
        ix.split_probe = True
        d3, i3 = ix.search(q, 100, 8, chunk=max(1, len(q) // 3 + 1))
        ok = ok and np.array_equal(i3, i) and d3.tobytes() == d.tobytes()
        ix.close()  # releases the graph before the process group goes
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_nccl():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get() for _ in range(2))
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    assert res == [(0, True), (1, True)]
