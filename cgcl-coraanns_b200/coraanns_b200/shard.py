"""Cluster-sharded search over several GPUs: one process and one engine per GPU.

The index is split by IVF cluster (``shard_plan``: longest-processing-time on cluster sizes,
the same plan on every rank); each engine keeps its clusters' codes and every centroid, so
each rank probes exactly as an unsharded engine would and scans only what it owns. A search
is three engine calls with two all-gathers between them, which this module runs over a
``torch.distributed`` process group (NCCL on GPUs):

    begin  -> all-gather each shard's k smallest vanguard seed keys -> global threshold T1
    resume -> all-gather each shard's top-k keys (+ its device error word)
    end    -> top-k of all shards

By default (``split_probe``) the probing is also split: each shard runs the probe GEMM and
the exact top-nprobe for its slice of the queries only, and a first all-gather of the probe
lists precedes ``begin`` (``probe -> all-gather -> begin_probed``).

The result equals an unsharded search of the whole index bit for bit (the reference searches
on one GPU only; this layer has no counterpart there).

``run_sharded_search`` is written against a small backend protocol (``begin / resume /
end`` + an ``exchange`` callable) so that the same orchestration drives the CUDA engine and,
in the CPU tests, the oracle.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import HybridIndex, LogicError, _check, _lib

KEY_MAX = np.uint64(0xFFFFFFFFFFFFFFFF)


def shard_plan(sizes, world: int) -> np.ndarray:
    """owner[c] = shard of cluster c (the engine's own plan, cora_shard_plan)."""
    s = np.ascontiguousarray(sizes, np.uint64)
    out = np.empty(s.shape[0], np.int32)
    _check(_lib.cora_shard_plan(s.ctypes.data_as(C.c_void_p), s.shape[0], int(world),
                                out.ctypes.data_as(C.c_void_p)))
    return out


def shard_search_data(sd: dict, owner: np.ndarray, rank: int) -> dict:
    """The SearchData-layout arrays of one shard (what a sharded engine keeps): every
    centroid, the owned clusters' vectors in their order, size 0 for the other clusters."""
    sizes = np.asarray(sd["sizes"], np.uint64).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    W = int(sd["D"]) // 32
    keep = np.flatnonzero(owner == rank)
    rows = np.concatenate([np.arange(starts[c], starts[c] + sizes[c]) for c in keep]) \
        if len(keep) else np.zeros(0, np.int64)
    short = np.asarray(sd["short_data"], np.uint32)
    # a cluster's 1-bit block is contiguous (word-major inside the cluster)
    short_parts = [short[starts[c] * W:(starts[c] + sizes[c]) * W] for c in keep]
    lc = np.asarray(sd["long_codes"], np.uint8).reshape(int(sd["num"]), -1)
    out = dict(sd)
    out.update(
        num=int(rows.shape[0]),
        short_data=np.concatenate(short_parts) if short_parts else np.zeros(0, np.uint32),
        short_factors=np.asarray(sd["short_factors"], np.float32).reshape(-1, 3)[rows],
        long_codes=lc[rows].reshape(-1),
        ex_factors=np.asarray(sd["ex_factors"], np.float32).reshape(-1, 2)[rows],
        ids=np.asarray(sd["ids"], np.uint32)[rows],
        sizes=np.where(owner == rank, sizes, 0).astype(np.uint64),
    )
    out.pop("bits", None)
    return out


def exchange_words(nq: int, k: int) -> int:
    """u64 words of one shard's exchange buffer: k keys per query + one status word."""
    return int(_lib.cora_shard_exchange_words(nq, k))


def torch_exchange(group=None):
    """All-gather over a torch.distributed group, ordered on torch's current stream."""
    import torch.distributed as dist

    def exchange(send, recv):
        dist.all_gather_into_tensor(recv, send, group=group)
    return exchange


def probe_words(nq: int, nprobe: int, world: int) -> int:
    """u64 words of one shard's probe-exchange buffer (its slice of the probe lists + one
    status word)."""
    return int(_lib.cora_shard_probe_words(nq, nprobe, world))


def run_sharded_search(backend, exchange, queries, nq, k, nprobe, out_d, out_i,
                       split_probe=False):
    """One search across all shards: every rank calls this with the same arguments. With
    split_probe each shard probes only its slice of the queries and a first all-gather
    exchanges the probe lists (backend.probe / begin_probed)."""
    send, recv = backend.buffers(nq, k)
    if split_probe:
        psend, precv = backend.probe_buffers(nq, nprobe)
        backend.probe(queries, nq, k, nprobe, psend)
        exchange(psend, precv)
        backend.begin_probed(precv, send)
    else:
        backend.begin(queries, nq, k, nprobe, send)
    exchange(send, recv)
    backend.resume(recv, send)
    exchange(send, recv)
    backend.end(recv, out_d, out_i)


def manifest_mismatch(manifests) -> str | None:
    """Why the shards' (rank, world, nlist, dim, padded_dim, clusters held) rows do not form
    one consistent sharding of one index, or None."""
    m = np.asarray(manifests, np.int64)
    world = int(m[0, 1])
    if len(m) != world or not (m[:, 1] == world).all():
        return f"world sizes differ: {m[:, 1].tolist()} across {len(m)} ranks"
    if sorted(m[:, 0].tolist()) != list(range(world)):
        return f"shard ranks are not 0..{world - 1}: {m[:, 0].tolist()}"
    for col, name in ((2, "nlist"), (3, "dim"), (4, "padded_dim")):
        if not (m[:, col] == m[0, col]).all():
            return f"{name} differs across shards: {m[:, col].tolist()}"
    if int(m[:, 5].sum()) != int(m[0, 2]):
        return f"shards hold {int(m[:, 5].sum())} clusters in total, the index has {int(m[0, 2])}"
    return None


class ShardedIndex:
    """One shard of a cluster-sharded index on this process's GPU, searched together with the
    other ranks of `group` (torch.distributed, NCCL). Every rank loads the same index and
    calls search with the same queries and arguments."""

    def __init__(self, device: int, group=None, split_probe: bool = True):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.engine = HybridIndex(device)
        self.engine.shard_configure(self.rank, self.world)
        self.device = device
        # probing split by query over the shards (an extra all-gather of probe lists); the
        # probing stage then costs each shard 1 / world of its single-GPU time
        self.split_probe = split_probe and self.world > 1
        self._bufs = None
        self._pbufs = None
        self._stream = None
        self._graph = None
        self.exchange = torch_exchange(group)

    # loading: the engine keeps only this rank's clusters
    def load_index_file(self, path):
        self.engine.load_index_file(path)
        self._verify()

    def load_search_data(self, sd):
        self.engine.load_search_data(sd)
        self._verify()

    def load_shard_arrays(self, sd_local, global_sizes):
        """This rank's clusters only (shard_search_data's layout, built or read by this rank
        alone) and the whole index's cluster sizes."""
        self.engine.load_shard_arrays(sd_local, global_sizes)
        self._verify()

    def _verify(self):
        import torch
        import torch.distributed as dist
        info, shape = self.engine.shard_info(), self.engine.index_info()
        row = torch.tensor([info["rank"], info["world"], shape["nlist"], shape["dim"],
                            shape["padded_dim"], info["clusters"]], dtype=torch.int64,
                           device=f"cuda:{self.device}")
        rows = torch.empty((self.world, 6), dtype=torch.int64, device=row.device)
        dist.all_gather_into_tensor(rows, row, group=self.group)
        why = manifest_mismatch(rows.cpu().numpy())
        if why:
            raise LogicError(f"inconsistent shards: {why}")

    def prepare_workspace(self, max_queries, max_topk, max_nprobe):
        import torch
        self.engine.prepare_workspace(max_queries, max_topk, max_nprobe)
        w = exchange_words(max_queries, max_topk)
        dev = f"cuda:{self.device}"
        self._bufs = (torch.empty(w, dtype=torch.int64, device=dev),
                      torch.empty(self.world * w, dtype=torch.int64, device=dev))
        pw = probe_words(max_queries, max_nprobe, self.world)
        self._pbufs = (torch.empty(pw, dtype=torch.int64, device=dev),
                       torch.empty(self.world * pw, dtype=torch.int64, device=dev))

    # backend protocol of run_sharded_search
    def buffers(self, nq, k):
        if self._bufs is None:
            raise LogicError("prepare workspace before searching")
        w = exchange_words(nq, k)
        return self._bufs[0][:w], self._bufs[1][:self.world * w]

    def probe_buffers(self, nq, nprobe):
        if self._pbufs is None:
            raise LogicError("prepare workspace before searching")
        w = probe_words(nq, nprobe, self.world)
        return self._pbufs[0][:w], self._pbufs[1][:self.world * w]

    def probe(self, queries, nq, k, nprobe, send):
        import torch
        self.engine.shard_search_probe(queries.data_ptr(), nq, k, nprobe, send.data_ptr(),
                                       torch.cuda.current_stream(self.device).cuda_stream)

    def begin_probed(self, recv, send):
        self.engine.shard_search_begin_probed(recv.data_ptr(), send.data_ptr())

    def begin(self, queries, nq, k, nprobe, send):
        import torch
        self.engine.shard_search_begin(queries.data_ptr(), nq, k, nprobe, send.data_ptr(),
                                       torch.cuda.current_stream(self.device).cuda_stream)

    def resume(self, recv, send):
        self.engine.shard_search_resume(recv.data_ptr(), send.data_ptr())

    def end(self, recv, out_d, out_i):
        self.engine.shard_search_end(recv.data_ptr(), out_d.data_ptr(), out_i.data_ptr())

    def _run_chunks(self, queries, k, nprobe, out_d, out_i, chunk):
        nq = queries.shape[0]
        step = nq if not chunk else int(chunk)
        for a in range(0, nq, step):
            b = min(nq, a + step)
            run_sharded_search(self, self.exchange, queries[a:b], b - a, k, nprobe, out_d[a:b],
                               out_i[a:b], self.split_probe)

    def search_device(self, queries, k, nprobe, out_d, out_i, chunk=None):
        """Device tensors, ordered after torch's current stream and before its later work;
        not synchronised. The search and its all-gathers run on this index's own stream
        (the engine's launches and NCCL's must share one non-default stream). `chunk`: search
        the batch in slices of at most that many queries (the shape limit queries x nlist
        < 2^31, as the reference's --query-chunk)."""
        import torch
        if self._stream is None:
            self._stream = torch.cuda.Stream(self.device)
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self._run_chunks(queries, k, nprobe, out_d, out_i, chunk)
        cur.wait_stream(self._stream)

    def capture(self, queries, k, nprobe, out_d, out_i, chunk=None):
        """Captures one whole sharded search (the engine's launches and both NCCL
        all-gathers) into a CUDA graph on this rank, for replay(); every rank captures the
        same search. The buffers are baked in: replay() searches `queries` into out_d / out_i
        as they hold at replay time. Run one eager search first (communicator set-up), and
        release the graph (release_graph / close) before the process group is destroyed."""
        import torch
        self.release_graph()
        g = torch.cuda.CUDAGraph()
        if self._stream is None:
            self._stream = torch.cuda.Stream(self.device)
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(g, stream=self._stream, capture_error_mode="relaxed"):
            self._run_chunks(queries, k, nprobe, out_d, out_i, chunk)
        self._graph = g

    def replay(self):
        """Replays the captured search on this index's stream, ordered after torch's current
        stream and before its later work; not synchronised."""
        import torch
        if self._graph is None:
            raise LogicError("capture a search before replaying it")
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self._graph.replay()
        cur.wait_stream(self._stream)

    def release_graph(self):
        if self._graph is not None:
            self._graph.reset()
            self._graph = None

    def search(self, h_queries, k, nprobe, chunk=None):
        """Host arrays in and out (queries copied to this rank's GPU)."""
        import torch
        q = torch.from_numpy(np.ascontiguousarray(h_queries, np.float32)).to(
            f"cuda:{self.device}", non_blocking=True)
        out_d = torch.empty((q.shape[0], k), dtype=torch.float32, device=q.device)
        out_i = torch.empty((q.shape[0], k), dtype=torch.int32, device=q.device)
        self.search_device(q, k, nprobe, out_d, out_i, chunk)
        d, i = out_d.cpu().numpy(), out_i.cpu().numpy().view(np.uint32)
        self.engine.check_device()
        return d, i

    def close(self):
        self.release_graph()
        self.engine.close()
