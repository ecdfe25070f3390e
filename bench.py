#!/usr/bin/env python3
"""Benchmark: QPS at recall@10 >= 0.95 of the IVF-RaBitQ search hot path on B200.

Workload (the single-GPU configuration the metric is quoted on):
10M float32 vectors, d = 96 (padded 128), 4096-component Gaussian mixture (centres
N(0, 1), sigma 0.25), L2, nlist 4096, 8-bit RaBitQ (1 + 7 ex bits), 10,000 queries
(mixture + N(0, 0.05) noise), topk 10, nprobe swept over 8..128; the reported nprobe is
the smallest whose distance-aware recall@10 (recall.hpp semantics) is >= 0.95.
Data are seeded synthetic stand-ins of that shape; the IVF partition is 2 Lloyd
iterations from the generating centres; the index is built on the GPU by
coraanns_b200.builder (the reference quantizer's "faster" mode).

One step = one search of the whole 10K-query batch. `value` times K steps with the
queries resident in HBM (CUDA events on the search stream, max over ranks); `e2e` times the
public host API (cora_search: pinned host queries -> HBM -> results back to host).
`--impl reference` times the reference's own CPU search (IVF::search, the rabitq_cpu loop,
compiled from the reference source into oracle/_ref) on the same index with every host
thread, on a bounded query sample per step.

Multi-GPU (torchrun, one process per GPU): N GPUs form N / S copies of the index, each copy
cluster-sharded over S GPUs (coraanns_b200.shard: every shard probes all centroids and scans
the clusters it owns; the shards' vanguard seed keys, which give the global pruning
threshold, and then their top-k keys are exchanged by NCCL all-gathers and merged). Each
copy answers its own 10K-query batch (queries are independent units: no collective between
copies), so the per-GPU work is fixed as N grows (weak scaling; strong only when a single
copy spans every GPU). S defaults to the fewest GPUs whose memory holds the index (1 for
config 2: every GPU holds a full copy and no collective runs on the data path); `--shards S`
forces cluster sharding. `value` is queries/s of the whole job.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "cgcl-coraanns_b200"), str(ROOT / "oracle")]

CONFIGS = {
    # name: N, dim, nlist, nq, sigma, qnoise, k, nprobes, seed
    "cfg2": dict(n=10_000_000, dim=96, nlist=4096, nq=10_000, sigma=0.25, qnoise=0.05, k=10,
                 nprobes=[8, 12, 16, 24, 32, 48, 64, 96, 128], seed=20261202),
    "demo": dict(n=4096, dim=128, nlist=16, nq=100, sigma=0.3, qnoise=0.05, k=10,
                 nprobes=[4, 8, 16], seed=20261201),
    "small": dict(n=1_000_000, dim=96, nlist=1024, nq=10_000, sigma=0.25, qnoise=0.05, k=10,
                  nprobes=[8, 16, 32, 64], seed=20261205),
    # profiling case: codes (5M x 32 B) larger than L2, a few GB on the device in total
    "medium": dict(n=5_000_000, dim=96, nlist=2048, nq=10_000, sigma=0.25, qnoise=0.05, k=10,
                   nprobes=[8], seed=20261206),
}
TARGET_RECALL = 0.95

# Configurations too large to hold as raw vectors: generated chunk by chunk from counter-based
# seeds (coraanns_b200.synthetic) and built in two streaming passes; one GPU, the index
# staged in host memory. BASELINE configs 4 and 3 (inner product on unit vectors).
STREAM_CONFIGS = {
    "cfg4": dict(n=88_000_000, dim=768, nlist=32768, nq=10_000, sigma=0.2, qnoise=0.05, k=100,
                 nprobes=[32, 48, 64, 96, 128, 192, 256, 384, 512], seed=20261204, metric=1,
                 zipf=None, vanguard=5),
    # Zipf(1.1) component weights: k-means starts from data samples, so heavy components get
    # several centroids (cluster sizes stay heavy-tailed)
    "cfg3": dict(n=100_000_000, dim=768, nlist=65536, nq=10_000, sigma=0.25, qnoise=0.05, k=10,
                 nprobes=[16, 24, 32, 48, 64, 96, 128, 192, 256], seed=20261203, metric=1,
                 zipf=1.1, vanguard=5, init="sample", queue=1 << 31),
    # a small case of the same shape (tests of the streamed path, profiling)
    "cfg4s": dict(n=4_000_000, dim=768, nlist=2048, nq=2000, sigma=0.2, qnoise=0.05, k=100,
                  nprobes=[16, 32, 64], seed=20261208, metric=1, zipf=None, vanguard=5),
    # config 4's probing stage (10K queries against 32768 centroids of d768) over a small
    # base (profiling the rotation, probe GEMM and probe selection at full size)
    "cfg4p": dict(n=4_000_000, dim=768, nlist=32768, nq=10_000, sigma=0.2, qnoise=0.05, k=100,
                  nprobes=[32], seed=20261209, metric=1, zipf=None, vanguard=5),
}

# Configurations generated per shard under torchrun (one rank per GPU): the clusters are the
# mixture's components, each rank generates and quantises only the clusters cora_shard_plan
# gives it, and the search runs cluster-sharded over all ranks.
SHARD_GEN_CONFIGS = {
    "cfg5": dict(n=1_000_000_000, dim=96, nlist=262_144, sigma=0.25, qnoise=0.05, nq=10_000,
                 k=10, nprobes=[64, 128, 256, 512, 1024], seed=20261205),
    # a small case of the same construction (the path's check at 1-2 GPUs)
    "cfg5s": dict(n=40_000_000, dim=96, nlist=16_384, sigma=0.25, qnoise=0.05, nq=10_000,
                  k=10, nprobes=[16, 32, 64, 128], seed=20261206),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------------
# data, partition, ground truth (GPU tooling, torch)
# ------------------------------------------------------------------------------------
def make_data(cfg, dev):
    import torch
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    centres = torch.randn(cfg["nlist"], cfg["dim"], generator=g, device=dev)
    base = torch.empty(cfg["n"], cfg["dim"], device=dev)
    chunk = 1 << 21
    for s in range(0, cfg["n"], chunk):
        e = min(cfg["n"], s + chunk)
        lab = torch.randint(0, cfg["nlist"], (e - s,), generator=g, device=dev)
        base[s:e] = centres[lab] + cfg["sigma"] * torch.randn(e - s, cfg["dim"], generator=g, device=dev)
    qlab = torch.randint(0, cfg["nlist"], (cfg["nq"],), generator=g, device=dev)
    q = (centres[qlab] + cfg["sigma"] * torch.randn(cfg["nq"], cfg["dim"], generator=g, device=dev)
         + cfg["qnoise"] * torch.randn(cfg["nq"], cfg["dim"], generator=g, device=dev))
    return centres, base, q.contiguous()


def make_queries(centres, cfg, n, seed, dev):
    """Another batch of n queries from the same mixture (a replica's own batch)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    qlab = torch.randint(0, cfg["nlist"], (n,), generator=g, device=dev)
    q = (centres[qlab] + cfg["sigma"] * torch.randn(n, cfg["dim"], generator=g, device=dev)
         + cfg["qnoise"] * torch.randn(n, cfg["dim"], generator=g, device=dev))
    return q.contiguous()


def assign(base, cent):
    import torch
    out = torch.empty(base.shape[0], dtype=torch.int64, device=base.device)
    cn = (cent * cent).sum(1)
    for s in range(0, base.shape[0], 1 << 20):
        x = base[s:s + (1 << 20)]
        out[s:s + x.shape[0]] = (cn[None, :] - 2 * x @ cent.T).argmin(1)
    return out


def kmeans(base, init, iters=2):
    import torch
    c = init.clone()
    for _ in range(iters):
        a = assign(base, c)
        sums = torch.zeros_like(c).index_add_(0, a, base)
        cnt = torch.bincount(a, minlength=c.shape[0]).float()
        nz = cnt > 0
        c[nz] = sums[nz] / cnt[nz, None]
    return c, assign(base, c)


def ground_truth(base, q, k):
    """Exact top-k by (fp64 distance, id): fp32 filter keeping 64 candidates per query,
    then fp64 recompute (tools/data/generate_gt_gpu.py:56-69,114-119 of the reference)."""
    import torch
    keep = 64
    bn = (base * base).sum(1)
    best_d = torch.full((q.shape[0], keep), float("inf"), device=q.device)
    best_i = torch.zeros((q.shape[0], keep), dtype=torch.int64, device=q.device)
    for s in range(0, base.shape[0], 1 << 20):
        x = base[s:s + (1 << 20)]
        d = bn[s:s + x.shape[0]][None, :] - 2 * q @ x.T
        vd, vi = torch.topk(d, keep, dim=1, largest=False)
        cd = torch.cat([best_d, vd], 1)
        ci = torch.cat([best_i, vi + s], 1)
        o = torch.topk(cd, keep, dim=1, largest=False).indices
        best_d, best_i = torch.gather(cd, 1, o), torch.gather(ci, 1, o)
    ex = ((base[best_i].double() - q[:, None, :].double()) ** 2).sum(2)
    # lexicographic (distance, id): stable sort by id, then stable sort by distance
    order_id = torch.argsort(best_i, dim=1, stable=True)
    ex, best_i = torch.gather(ex, 1, order_id), torch.gather(best_i, 1, order_id)
    order = torch.argsort(ex, dim=1, stable=True)[:, :k]
    return torch.gather(best_i, 1, order), torch.gather(ex, 1, order)


def recall_at_k(base, q, gt_ids, gt_d, res_ids, k):
    """Distance-aware recall@k (include/coraanns/benchmark/recall.hpp:133-190)."""
    import torch
    r = torch.as_tensor(res_ids.astype(np.int64), device=q.device)[:, :k]
    valid = r < base.shape[0]
    rc = torch.where(valid, r, torch.zeros_like(r))
    in_gt = (rc[:, :, None] == gt_ids[:, None, :k]).any(2)
    d = ((base[rc].double() - q[:, None, :].double()) ** 2).sum(2)
    ok = valid & (in_gt | (d <= gt_d[:, k - 1:k]))
    # repeated ids count once
    srt, _ = torch.sort(torch.where(ok, rc, torch.full_like(rc, -1)), dim=1)
    dup = torch.zeros_like(ok)
    dup[:, 1:] = (srt[:, 1:] == srt[:, :-1]) & (srt[:, 1:] >= 0)
    hits = (srt >= 0).sum() - dup.sum()
    return float(hits) / (q.shape[0] * k)


# ------------------------------------------------------------------------------------
# measurement helpers
# ------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def apply_tuning(engine, pairs):
    """cora_set_tuning for each KEY=VALUE of --tuning."""
    for kv in pairs:
        key, _, val = kv.partition("=")
        engine.set_tuning(key, int(val))


def launches_per_search(nprobe, k, mode, shards, estimator, metric, split_probe=False):
    """Kernels one search launches: rotation, probe GEMM, probe selection (warp kernel + its
    block fallback when nprobe <= 32), seed refine, threshold, main grouping (4), main scan,
    refine, merge (threshold and final top-k: warp kernel + block fallback each when
    k <= 32); with stored vanguard lows also vanguard grouping (4), lows scan, seed selection
    (warp + block fallback when keep <= 128) and the lows filter (pair list + filter), else
    one vanguard rescan; +2 exchange steps (gather_threshold / gather_merge) when sharded,
    +2 more (pack / unpack of the probe lists) with the probing split by query;
    +1 LUT build for the LUT estimator; +1 additive-term kernel for inner product."""
    sel = 2 if nprobe <= 32 else 1
    vsel = 2 if max(k, 20) <= 128 else 1
    topk = 2 if k <= 32 else 1
    return (9 + sel + 2 * topk + ((7 + vsel) if mode == 1 else 1)
            + (2 if shards > 1 else 0) + (2 if shards > 1 and split_probe else 0)
            + (1 if estimator == "lut" else 0) + (1 if metric else 0))



def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    return 6650.0, "fallback (6.65 TB/s)"


def profiled_traffic(config, estimator):
    """DRAM bytes (read + write) of one launch of the scan's lows pass (the dominant kernel)
    with the given estimator, from the committed ncu summary of the full-size config-2
    workload (None for other configs, or before that capture exists)."""
    p = ROOT / "profiles" / "scan_kernel_cfg2_dram.md"
    if config != "cfg2" or not p.exists():
        return None
    key = f"dram_bytes_lows_pass_full_size_{estimator}:"
    for line in p.read_text().splitlines():
        if line.startswith(key):
            return int(line.split(":")[1])
    return None


def cpu_reference_qps(index_path, q_np, k, nprobe, target_seconds=15.0, threads=None):
    """The reference's own CPU search (oracle/_ref IVF::search, rabitq_cpu loop) on a
    bounded sample, or the C oracle port when the reference harness is absent."""
    import py_oracle as po
    threads = threads or os.cpu_count() or 1
    if po.ref_available():
        ivf = po.RefIVF(index_path)
        run = lambda qs: ivf.search(qs, k, nprobe, threads=threads)  # noqa: E731
        kind = "reference"
    else:
        o = po.oracle_from_file(index_path)
        run = lambda qs: o.search(qs, k, nprobe, threads=threads)  # noqa: E731
        kind = "port"
    probe = q_np[:min(len(q_np), max(threads * 4, 256))]
    t = time.perf_counter()
    run(probe)
    per_q = max((time.perf_counter() - t) / len(probe), 1e-7)
    m = int(min(len(q_np), max(len(probe), target_seconds / per_q)))
    # repeat the sample (at most 20 times) so the measurement spans about target_seconds
    reps = int(max(1, min(20, target_seconds / (per_q * m))))
    sample = q_np[:m]
    t = time.perf_counter()
    for _ in range(reps):
        run(sample)
    dt = time.perf_counter() - t
    return dict(value=m * reps / dt, unit="queries/s", cores=threads, kind=kind,
                sample=f"{m} of the {len(q_np)} queries x {reps}, nprobe {nprobe}, topk {k}, "
                       f"{dt:.1f} s"), run


_OUT_FD = None


def redirect_stdout():
    """Route everything libraries print to stdout (e.g. NCCL's version banner) to stderr,
    so that the result line is the only thing on stdout."""
    global _OUT_FD
    sys.stdout.flush()
    _OUT_FD = os.dup(1)
    os.dup2(2, 1)


def emit(line: dict):
    data = (json.dumps(line) + "\n").encode()
    if _OUT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_OUT_FD, data)


def auto_shards(sd, world, dev) -> int:
    """Fewest GPUs per copy of the index that keep a copy under half of one GPU's memory
    (the rest is workspace); 1 when the index fits, so every GPU holds a full copy."""
    import torch
    n, D = int(sd["num"]), int(sd["D"])
    index_bytes = n * (D // 8 + 12 + D * 7 // 8 + 8 + 4) + int(sd["nlist"]) * D * 4
    budget = torch.cuda.get_device_properties(dev).total_memory // 2
    for s in range(1, world + 1):
        if world % s == 0 and index_bytes // s <= budget:
            return s
    return world


# ------------------------------------------------------------------------------------
# cluster-sharded sub-measurement (N > 1)
# ------------------------------------------------------------------------------------
def measure_sharded(args, sd, q, k, nprobe, kernel_type, eng_single, local, world, dev, total):
    """The same N GPUs as one cluster-sharded copy of the index answering one batch (the
    north star's multi-GPU layout; strong scaling): every rank loads its shard, the search's
    two exchanges are NCCL all-gathers, and the whole search (engine launches and both
    all-gathers) is also captured in one CUDA graph per rank and replayed. Reported beside
    the headline: QPS eager and replayed (max over ranks of the CUDA-event time), the
    single-GPU time of the same batch on each rank's own full copy, the strong-scaling
    efficiency t_single / (N t_sharded), bit-identity with the single-GPU result, and every
    rank's stage times (eager, with stage events)."""
    import torch
    import torch.distributed as dist
    from coraanns_b200.shard import ShardedIndex
    nq = q.shape[0]
    six = ShardedIndex(local)
    apply_tuning(six.engine, args.tuning)
    six.engine.set_ip_kernel_type(kernel_type)
    six.load_search_data(sd)
    six.prepare_workspace(nq, k, nprobe)
    od = torch.empty((nq, k), dtype=torch.float32, device=dev)
    oi = torch.empty((nq, k), dtype=torch.int32, device=dev)
    sd_ = torch.empty_like(od)
    si = torch.empty_like(oi)
    st = torch.cuda.Stream(dev)

    def single():
        eng_single.search_device(q.data_ptr(), nq, k, nprobe, sd_.data_ptr(), si.data_ptr(),
                                 st.cuda_stream)

    def timed(fn, reps):
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return total(e0.elapsed_time(e1) / reps, dist.ReduceOp.MAX)

    eager = lambda: six.search_device(q, k, nprobe, od, oi)  # noqa: E731
    cur = torch.cuda.current_stream(dev)
    st.wait_stream(cur)
    single()
    cur.wait_stream(st)
    for _ in range(args.warmup):
        eager()
    torch.cuda.synchronize()
    six.engine.check_device()
    eng_single.check_device()
    identical = bool(torch.equal(od, sd_) and torch.equal(oi, si))
    identical = total(1.0 if identical else 0.0, dist.ReduceOp.MIN) == 1.0

    def single_ordered():
        st.wait_stream(torch.cuda.current_stream(dev))
        single()
        torch.cuda.current_stream(dev).wait_stream(st)

    reps = max(args.steps, 20)
    ms_single = timed(single_ordered, reps)
    ms_eager = timed(eager, reps)
    six.capture(q, k, nprobe, od, oi)
    six.replay()
    torch.cuda.synchronize()
    ms_graph = timed(six.replay, reps)
    six.engine.check_device()
    same_graph = total(1.0 if (torch.equal(od, sd_) and torch.equal(oi, si)) else 0.0,
                       dist.ReduceOp.MIN) == 1.0
    six.release_graph()
    # stage times of every rank (eager launches with stage events)
    import coraanns_b200 as cb
    six.engine.set_profiling(True)
    eager()
    torch.cuda.synchronize()
    six.engine.stage_reset()
    for _ in range(5):
        eager()
    torch.cuda.synchronize()
    cnt, tot = six.engine.stage_totals()
    six.engine.set_profiling(False)
    mine = torch.tensor([tot[s] / max(cnt, 1) for s in cb.STAGES], dtype=torch.float64, device=dev)
    allr = torch.empty((world, len(cb.STAGES)), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(allr, mine)
    six.close()
    best = min(ms_eager, ms_graph)
    return dict(layout=f"one copy of the index, {world} cluster shards, {nq} queries",
                qps_eager=nq / (ms_eager / 1e3), qps_graph=nq / (ms_graph / 1e3),
                ms_eager=ms_eager, ms_graph=ms_graph, ms_single_gpu=ms_single,
                strong_scaling_efficiency=ms_single / (world * best),
                identical_to_single_gpu=identical and same_graph,
                stage_ms_per_rank=[dict(zip(cb.STAGES, map(float, r))) for r in allr.cpu().numpy()])


# ------------------------------------------------------------------------------------
# streamed configurations (one GPU)
# ------------------------------------------------------------------------------------
def run_stream(args, name, cfg):
    import torch
    import coraanns_b200 as cb
    from coraanns_b200 import synthetic
    import py_oracle as po

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    k, nq, metric = cfg["k"], cfg["nq"], cfg["metric"]
    t0 = time.time()
    mix = synthetic.Mixture(cfg["n"], cfg["dim"], cfg["nlist"], cfg["sigma"], cfg["seed"],
                            normalise=metric == 1, zipf_s=cfg["zipf"], device=dev)
    cent = synthetic.train_centroids(mix, cfg["nlist"], init=cfg.get("init", "centres"),
                                     sample=max(1 << 21, 64 * cfg["nlist"]))
    sd = synthetic.build_index_stream(mix, cent, metric=metric, seed=cfg["seed"], log=log)
    log(f"[bench] {name}: index built in {time.time() - t0:.1f}s")
    q = mix.queries(nq, cfg["qnoise"])
    t1 = time.time()
    gt_ids, gt_d = synthetic.ground_truth_stream(mix, q, k, metric=metric)
    log(f"[bench] ground truth in {time.time() - t1:.1f}s")
    q_np = q.cpu().numpy()
    torch.cuda.empty_cache()

    eng = cb.HybridIndex(0)
    apply_tuning(eng, args.tuning)
    eng.set_vanguard_size(cfg["vanguard"])
    # candidate records per search (16 B each); the Zipf configuration's heavy clusters
    # (largest ~150K vectors) need more than 2^30 / 10K per query
    eng.set_queue_capacity(cfg.get("queue", 1 << 28))
    t2 = time.time()
    eng.load_search_data(sd)
    eng.prepare_workspace(nq, k, max(cfg["nprobes"]))
    log(f"[bench] engine loaded in {time.time() - t2:.1f}s")
    stream = torch.cuda.Stream(dev)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_i = torch.empty((nq, k), dtype=torch.int32, device=dev)

    def search_dev(npb):
        eng.search_device(q.data_ptr(), nq, k, npb, out_d.data_ptr(), out_i.data_ptr(),
                          stream.cuda_stream)

    def quick_ms(npb, reps=3):
        search_dev(npb)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            search_dev(npb)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    # every (estimator, nprobe) result of the sweep, scored exactly in one pass
    estimators = {"bitwise": cb.KernelType.Bitwise, "lut": cb.KernelType.Lut4Bit}
    if args.estimator != "auto":
        estimators = {args.estimator: estimators[args.estimator]}
    nprobes = [args.nprobe] if args.nprobe else cfg["nprobes"]
    runs, results, overflow = [], [], {}
    for ename, kt in estimators.items():
        eng.set_ip_kernel_type(kt)
        for npb in nprobes:
            search_dev(npb)
            torch.cuda.synchronize()
            try:
                eng.check_device()
            except cb.CoraRuntimeError as ex:  # candidates beyond the HBM queue: larger
                overflow[ename] = dict(nprobe=npb, error=str(ex))  # nprobes would be too
                break
            runs.append((ename, npb))
            results.append(out_i.to(torch.int64).clone())
    eng.set_ip_kernel_type(cb.KernelType.Bitwise)
    allr = torch.cat(results, 1)
    t3 = time.time()
    exact = synthetic.exact_scores(mix, q, allr, metric)
    log(f"[bench] exact rescoring of the sweep in {time.time() - t3:.1f}s")
    sweeps, candidates = {}, {}
    for j, (ename, npb) in enumerate(runs):
        r = synthetic.distance_recall(gt_ids, gt_d, results[j], exact[:, j * k:(j + 1) * k], k)
        sweeps.setdefault(ename, {})[npb] = round(r, 4)
    for ename, kt in estimators.items():
        for npb in nprobes:
            if sweeps.get(ename, {}).get(npb, 0.0) >= TARGET_RECALL:
                eng.set_ip_kernel_type(kt)
                candidates[ename] = dict(nprobe=npb, recall=sweeps[ename][npb], ms=quick_ms(npb))
                break
    if candidates:
        estimator = min(candidates, key=lambda n: candidates[n]["ms"])
        chosen = candidates[estimator]["nprobe"]
    else:
        estimator, chosen = next(iter(estimators)), nprobes[-1]
    eng.set_ip_kernel_type(estimators[estimator])
    log(f"[bench] recall sweeps {sweeps} -> {estimator} estimator, nprobe {chosen}")

    search_dev(chosen)
    torch.cuda.synchronize()
    eng.check_device()
    probes = eng.debug("probe_ids", nq, chosen)
    refined = eng.get_last_submitted_count()
    sizes = sd["sizes"].astype(np.int64)
    D = int(sd["D"])
    veff = min(max(eng.get_vanguard_size(), 1), chosen)
    lows_bytes = int(sizes[probes[:, :veff]].sum()) * (D // 8 + 12)
    scan_bytes = int(sizes[probes].sum()) * (D // 8 + 12)

    for _ in range(args.warmup):
        search_dev(chosen)
    eng.check_device()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_repeat():
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            search_dev(chosen)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / args.steps

    with ClockSampler(0) as clk:
        per_step = [timed_repeat()]
        want = int(1000.0 * args.min_seconds / max(per_step[0] * args.steps, 1e-3)) + 1
        for _ in range(0 if args.min_seconds <= 0 else max(2, min(50, want - 1))):
            per_step.append(timed_repeat())
    eng.check_device()
    rep_ms = np.array(per_step)
    ms = float(np.median(rep_ms))
    qps = nq / (ms / 1e3)

    eng.set_profiling(True)
    search_dev(chosen)
    eng.check_device()
    eng.stage_reset()
    for _ in range(3):
        search_dev(chosen)
    torch.cuda.synchronize()
    eng.check_device()
    count, stage_tot = eng.stage_totals()
    stage_avg = {st: v / max(count, 1) for st, v in stage_tot.items()}
    eng.set_profiling(False)

    qh = torch.empty((nq, cfg["dim"]), dtype=torch.float32, pin_memory=True)
    qh.copy_(q.cpu())
    qh_np = qh.numpy()
    od = torch.empty((nq, k), dtype=torch.float32, pin_memory=True).numpy()
    oi = torch.empty((nq, k), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    eng.reset_buffer(qh_np)
    for _ in range(args.warmup):
        eng.search(qh_np, k, chosen, out=(od, oi))
    e2e_steps = args.steps * len(rep_ms)
    t = time.perf_counter()
    for _ in range(e2e_steps):
        eng.search(qh_np, k, chosen, out=(od, oi))
    e2e_qps = nq / ((time.perf_counter() - t) / e2e_steps)

    peak, peak_src = measured_peaks()
    mode = eng.get_vanguard_mode()
    if mode == 1:
        kern_ms, kern_bytes = stage_avg["vanguard_scan"], lows_bytes
        kern = "scan_kernel lows pass (vanguard pairs)"
    else:
        kern_ms = stage_avg["vanguard_scan"] + stage_avg["main_scan"]
        kern_bytes, kern = scan_bytes, "scan_kernel (vanguard rescan + main pass)"
    achieved = kern_bytes / (kern_ms / 1e3) / 1e9 if kern_ms > 0 else None
    b_search = scan_bytes + refined * (7 * D // 8 + 12)
    roofline = dict(bound="hbm", kernel=kern, achieved=achieved, peak=peak, unit="GB/s",
                    frac=(achieved / peak) if achieved else None, traffic=None,
                    peak_source=peak_src, algorithmic_bytes_per_launch=kern_bytes,
                    launch_ms=kern_ms,
                    search_per_query=dict(bytes_per_query=b_search / nq,
                                          achieved=b_search / (ms / 1e3) / 1e9,
                                          frac=b_search / (ms / 1e3) / 1e9 / peak),
                    note="bytes = n_c*(D/8+12) per (query, probed cluster) of the launch")

    # CPU baseline: the C oracle (a port of the reference's arithmetic) on the host arrays
    # with every host thread, on a bounded query sample (the reference's own CPU search needs
    # the index as a file with an hnswlib sidecar, which cannot be written at this size here)
    cpu_base = None
    if not args.no_cpu_baseline:
        o = po.OracleIndex(sd, lut=estimator == "lut")
        threads = os.cpu_count() or 1
        probe_n = max(threads, 16)
        tt = time.perf_counter()
        o.search(q_np[:probe_n], k, chosen, vanguard=cfg["vanguard"], threads=threads)
        per_q = max((time.perf_counter() - tt) / probe_n, 1e-6)
        m = int(min(nq, max(probe_n, 20.0 / per_q)))
        tt = time.perf_counter()
        o.search(q_np[:m], k, chosen, vanguard=cfg["vanguard"], threads=threads)
        dt = time.perf_counter() - tt
        cpu_base = dict(value=m / dt, unit="queries/s", cores=threads, kind="port",
                        sample=f"{m} of the {nq} queries, nprobe {chosen}, topk {k}, {dt:.1f} s "
                               "(C oracle over the in-memory index)")

    line = dict(
        metric=f"QPS at recall@{k}>=0.95 (IVF-RaBitQ search)", value=qps, unit="queries/s",
        n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms, higher_is_better=True,
        scaling="weak", vs_baseline=None,
        dtype="i8+f32" if estimator == "bitwise" else "f16+f32",
        data=f"synthetic (seeded Gaussian mixture, BASELINE {name[:4]} shape, generated per chunk)",
        config=dict(workload=f"{name}: {cfg['n']} x d{cfg['dim']} "
                             f"{'inner product (unit vectors)' if metric else 'L2'}, "
                             f"nlist {cfg['nlist']}, 8-bit RaBitQ, {nq} queries, topk {k}"
                             + (f", Zipf({cfg['zipf']}) component weights" if cfg["zipf"] else ""),
                    nprobe=chosen, recall=sweeps.get(estimator, {}).get(chosen),
                    estimator=estimator, recall_sweeps=sweeps, qualifying=candidates,
                    sweep_stopped_by_queue_overflow=overflow or None,
                    vanguard=cfg["vanguard"], vanguard_mode="lows" if mode == 1 else "rescan",
                    candidates_per_query=refined / nq, stage_ms=stage_avg,
                    largest_cluster=int(sizes.max()), timed_repeats=len(rep_ms),
                    l2_flush="inputs exceed L2 (index codes > 126 MB)"),
        roofline=roofline, cpu_baseline=cpu_base,
        e2e=dict(value=e2e_qps, unit="queries/s", h2d_bytes_per_step=nq * cfg["dim"] * 4,
                 d2h_bytes_per_step=nq * k * 8),
        gpu_launches=launches_per_search(chosen, k, mode, 1, estimator, metric) * args.steps
        * len(rep_ms), clocks=clk.summary())
    emit(line)
    eng.close()


# ------------------------------------------------------------------------------------
# per-shard generated configurations (one copy of the index over all ranks)
# ------------------------------------------------------------------------------------
def run_shard_gen(args, name, cfg):
    """BASELINE config 5's construction: every rank generates, quantises and loads only its
    own clusters (cora_load_shard_arrays), so no host holds the whole index; ranks build in
    waves sized to the host's memory. The ground truth is the merge of every shard's exact
    top-k; recall is distance-aware with exact scores gathered from the owning shards. The
    search is one cluster-sharded copy over all ranks answering one batch (strong scaling),
    replayed from one CUDA graph per rank (engine launches and both NCCL all-gathers); QPS is
    the batch over the max-over-ranks device time."""
    import gc
    import psutil
    import torch
    import torch.distributed as dist
    import coraanns_b200 as cb
    from coraanns_b200 import synthetic
    from coraanns_b200.shard import ShardedIndex, shard_plan

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    timeout = __import__("datetime").timedelta(seconds=900)
    if "MASTER_ADDR" in os.environ:
        dist.init_process_group("nccl", timeout=timeout, device_id=dev)
    else:
        import socket
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1, timeout=timeout, device_id=dev)

    def total(x, op):
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    k, nq, nprobes = cfg["k"], cfg["nq"], list(cfg["nprobes"])
    if args.nprobe:
        nprobes = [args.nprobe]
    t0 = time.time()
    mix = synthetic.ComponentShards(cfg["n"], cfg["dim"], cfg["nlist"], cfg["sigma"],
                                    cfg["seed"], device=dev)
    owner = shard_plan(mix.counts, world)
    local_n = int(mix.counts[owner == rank].sum())
    per_rank = [total(local_n if r == rank else 0, dist.ReduceOp.SUM) for r in range(world)]
    host_need = max(per_rank) * synthetic.shard_bytes_per_vector(cfg["dim"])
    avail = total(psutil.virtual_memory().available if rank == 0 else 0, dist.ReduceOp.SUM)
    wave = max(1, min(world, int(0.5 * avail // max(host_need, 1))))
    six = ShardedIndex(local)
    apply_tuning(six.engine, args.tuning)
    for w in range((world + wave - 1) // wave):
        if rank // wave == w:
            sd = synthetic.build_shard(mix, owner, rank, metric=0, seed=cfg["seed"], log=log)
            six.engine.load_shard_arrays(sd, mix.counts)
            del sd
            gc.collect()
            torch.cuda.empty_cache()
        dist.barrier()
    six._verify()
    build_s = time.time() - t0
    log(f"[bench] {name}: {world} shards of {per_rank[0]:.0f}..{max(per_rank):.0f} vectors "
        f"built and loaded in {build_s:.1f}s (waves of {wave})")

    q = mix.queries(nq, cfg["qnoise"])
    q_np = q.cpu().numpy()
    t1 = time.time()
    li, ld = synthetic.ground_truth_shard(mix, owner, rank, q, k)
    gi = [torch.empty_like(li) for _ in range(world)]
    gd = [torch.empty_like(ld) for _ in range(world)]
    dist.all_gather(gi, li)
    dist.all_gather(gd, ld)
    gt_ids, gt_d = synthetic.merge_topk(torch.cat(gi, 1), torch.cat(gd, 1), k)
    log(f"[bench] ground truth (merged over shards) in {time.time() - t1:.1f}s")
    del gi, gd, li, ld
    gc.collect()
    torch.cuda.empty_cache()  # the ground truth's score blocks stay cached otherwise

    # the shape limit queries x nlist < 2^31 (validate_search_shape, as the reference's):
    # the batch is searched in equal query chunks (the reference CLI's --query-chunk)
    qmax = (2 ** 31 - 1) // cfg["nlist"]
    chunk = -(-nq // -(-nq // qmax))
    six.prepare_workspace(chunk, k, max(nprobes))
    od = torch.empty((nq, k), dtype=torch.float32, device=dev)
    oi = torch.empty((nq, k), dtype=torch.int32, device=dev)

    def recall_now():
        ids = oi.to(torch.int64)
        sc = synthetic.exact_scores_shard(mix, owner, rank, q, ids)
        dist.all_reduce(sc, op=dist.ReduceOp.MIN)
        return synthetic.distance_recall(gt_ids, gt_d, ids, sc, k)

    def timed(fn, reps):
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return total(e0.elapsed_time(e1) / reps, dist.ReduceOp.MAX)

    estimators = {"bitwise": cb.KernelType.Bitwise, "lut": cb.KernelType.Lut4Bit}
    if args.estimator != "auto":
        estimators = {args.estimator: estimators[args.estimator]}
    # per estimator: nprobe ascending up to the first that reaches the target, or until
    # the recall stops rising (two points within 0.001: more probes do not help)
    sweeps, candidates = {}, {}
    for ename, kt in estimators.items():
        six.engine.set_ip_kernel_type(kt)
        prev = -1.0
        for npb in nprobes:
            six.search_device(q, k, npb, od, oi, chunk)
            torch.cuda.synchronize()
            six.engine.check_device()
            r = recall_now()
            sweeps.setdefault(ename, {})[npb] = round(r, 4)
            if r >= TARGET_RECALL:
                ms = timed(lambda: six.search_device(q, k, npb, od, oi, chunk), 3)  # noqa: B023
                candidates[ename] = dict(nprobe=npb, recall=round(r, 4), ms=ms)
                break
            if r - prev < 1e-3:
                break
            prev = r
    if candidates:
        estimator = min(candidates, key=lambda n: candidates[n]["ms"])
        chosen = candidates[estimator]["nprobe"]
    else:
        estimator, chosen = next(iter(estimators)), nprobes[-1]
    six.engine.set_ip_kernel_type(estimators[estimator])
    log(f"[bench] recall sweeps {sweeps} -> {estimator} estimator, nprobe {chosen}")

    eager = lambda: six.search_device(q, k, chosen, od, oi, chunk)  # noqa: E731
    for _ in range(args.warmup):
        eager()
    torch.cuda.synchronize()
    six.engine.check_device()
    six.capture(q, k, chosen, od, oi, chunk)
    for _ in range(args.warmup):
        six.replay()
    torch.cuda.synchronize()
    six.engine.check_device()
    with ClockSampler(local) as clk:
        per_step = [timed(six.replay, args.steps)]
        want = int(1000.0 * args.min_seconds / max(per_step[0] * args.steps, 1e-3)) + 1
        for _ in range(0 if args.min_seconds <= 0 else max(2, min(50, want - 1))):
            per_step.append(timed(six.replay, args.steps))
    six.engine.check_device()
    six.release_graph()
    ms = float(np.median(per_step))
    qps = nq / (ms / 1e3)
    recall = recall_now()

    # stage times per rank (eager, stage events)
    six.engine.set_profiling(True)
    eager()
    torch.cuda.synchronize()
    six.engine.stage_reset()
    for _ in range(3):
        eager()
    torch.cuda.synchronize()
    cnt, tot = six.engine.stage_totals()
    six.engine.set_profiling(False)
    mine = torch.tensor([tot[s_] / max(cnt, 1) for s_ in cb.STAGES], dtype=torch.float64,
                        device=dev)
    allr = torch.empty((world, len(cb.STAGES)), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(allr, mine)
    stage_ranks = [dict(zip(cb.STAGES, map(float, r_))) for r_ in allr.cpu().numpy()]

    # end to end through the public API: host queries in, host results out, every step
    for _ in range(args.warmup):
        six.search(q_np, k, chosen, chunk)
    dist.barrier()
    e2e_steps = args.steps * len(per_step)
    tt = time.perf_counter()
    for _ in range(e2e_steps):
        six.search(q_np, k, chosen, chunk)
    e2e_s = total((time.perf_counter() - tt) / e2e_steps, dist.ReduceOp.MAX)

    # roofline of the lows pass on this rank: its vanguard pairs' clusters (the probe lists
    # of the last chunk, scaled to the batch)
    nlast = nq - (nq - 1) // chunk * chunk
    probes = six.engine.debug("probe_ids", nlast, chosen)
    veff = min(max(six.engine.get_vanguard_size(), 1), chosen)
    vg = probes[:, :veff]
    D = builder_padded(cfg["dim"])
    lows_bytes = int(int(mix.counts[vg][owner[vg] == rank].sum()) * (D // 8 + 12) * nq / nlast)
    nchunks = -(-nq // chunk)
    kern_ms = stage_ranks[rank]["vanguard_scan"] * nchunks  # stage times are per chunk search
    achieved = lows_bytes / (kern_ms / 1e3) / 1e9 if kern_ms > 0 else None
    peak, peak_src = measured_peaks()
    roof = dict(bound="hbm", kernel="scan_kernel lows pass (this rank's vanguard pairs)",
                achieved=achieved, peak=peak, unit="GB/s",
                frac=(achieved / peak) if achieved else None, traffic=None, peak_source=peak_src,
                algorithmic_bytes_per_launch=lows_bytes, launch_ms=kern_ms, rank=rank,
                note="bytes = n_c*(D/8+12) per (query, probed cluster) of the batch's lows "
                     "passes (one per query chunk)")
    roofs = [None] * world
    dist.all_gather_object(roofs, roof)
    mode = six.engine.get_vanguard_mode()
    per_search = launches_per_search(chosen, k, mode, world, estimator, 0,
                                     six.split_probe) * nchunks
    if rank == 0:
        line = dict(
            metric=f"QPS at recall@{k}>=0.95 (IVF-RaBitQ search)", value=qps, unit="queries/s",
            n_gpus=world, steps=args.steps, warmup=args.warmup, ms_per_step=ms,
            higher_is_better=True, scaling="strong", vs_baseline=None,
            dtype="i8+f32" if estimator == "bitwise" else "f16+f32",
            data=f"synthetic (seeded Gaussian mixture, BASELINE {name[:4]} shape, each shard's "
                 "clusters generated by its own rank)",
            config=dict(workload=f"{name}: {cfg['n']} x d{cfg['dim']} L2, nlist {cfg['nlist']} "
                                 f"(the mixture's components), 8-bit RaBitQ, {nq} queries, "
                                 f"topk {k}, cluster-sharded over {world} GPUs",
                        nprobe=chosen, recall=round(recall, 4), estimator=estimator,
                        recall_sweeps=sweeps, qualifying=candidates, shards=world,
                        vectors_per_shard=[int(v) for v in per_rank], build_s=round(build_s, 1),
                        build_waves=wave, timed_repeats=len(per_step), query_chunk=chunk,
                        stage_ms_per_rank=stage_ranks, stage_ms_are="per query-chunk search",
                        l2_flush="inputs exceed L2 (index codes > 126 MB)",
                        cpu_baseline_note="no host holds the whole index; the reference's CPU "
                                          "search is timed on configs 1-4"),
            roofline=roofs[0], roofline_per_rank=roofs, cpu_baseline=None,
            e2e=dict(value=nq / e2e_s, unit="queries/s", h2d_bytes_per_step=nq * cfg["dim"] * 4,
                     d2h_bytes_per_step=nq * k * 8),
            gpu_launches=per_search * args.steps * len(per_step), clocks=clk.summary())
        emit(line)
    six.close()
    dist.barrier()
    dist.destroy_process_group()


def builder_padded(dim):
    from coraanns_b200 import builder
    return builder.padded_dim(dim)


# ------------------------------------------------------------------------------------
# main
# ------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + sorted(STREAM_CONFIGS)
                    + sorted(SHARD_GEN_CONFIGS), default="cfg2")
    ap.add_argument("--nprobe", type=int, default=0, help="fix nprobe instead of sweeping")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shards", type=int, default=0,
                    help="GPUs per copy of the index (cluster shards); 0 = as memory requires")
    ap.add_argument("--estimator", choices=["auto", "bitwise", "lut"], default="auto",
                    help="the scan's estimator; auto times whichever of the reference's two "
                         "kernel types reaches the recall target fastest (forcing one also skips "
                         "the full-code side measurement: for short profiling runs)")
    ap.add_argument("--min-seconds", type=float, default=1.0,
                    help="repeat the timed K steps until they span this long (at least 3 "
                         "repeats when > 0; 0: one repeat, for profiling)")
    ap.add_argument("--tuning", action="append", default=[], metavar="KEY=VALUE",
                    help="engine tuning key (cora_set_tuning) applied to every engine, e.g. "
                         "refine_lanes=4; repeatable")
    ap.add_argument("--no-sharded", action="store_true",
                    help="with N > 1 GPUs, skip the cluster-sharded sub-measurement")
    ap.add_argument("--queries", type=int, default=0,
                    help="search only the first N queries of the batch (profiling a GPU's "
                         "slice of a multi-GPU run); 0 = the whole batch")
    args = ap.parse_args()
    redirect_stdout()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.config in SHARD_GEN_CONFIGS:
        if args.impl != "ours":
            emit({"impl": args.impl, "unavailable": f"{args.config}: no host holds the whole "
                                                    "index for the reference's CPU search"})
            return
        run_shard_gen(args, args.config, SHARD_GEN_CONFIGS[args.config])
        return
    if args.config in STREAM_CONFIGS:
        if int(os.environ.get("WORLD_SIZE", 1)) > 1 or args.impl != "ours":
            emit({"impl": args.impl, "unavailable": f"{args.config} runs on one GPU, ours only"})
            return
        run_stream(args, args.config, STREAM_CONFIGS[args.config])
        return

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = True
    cfg = CONFIGS[args.config]
    k = cfg["k"]

    if args.impl == "reference" and rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    t0 = time.time()
    centres, base, q = make_data(cfg, dev)
    if args.queries:
        cfg = dict(cfg, nq=min(args.queries, cfg["nq"]))
        q = q[:cfg["nq"]].contiguous()
    cent, lab = kmeans(base, centres)
    if world > 1:
        # every shard must cut the same partition: take rank 0's
        dist.broadcast(cent, 0)
        dist.broadcast(lab, 0)
    log(f"[bench] data + partition {time.time() - t0:.1f}s")
    # the builder is torch-only tooling; importing it does not map the search library, so
    # the reference arm below never loads libcoraanns_b200.so
    from coraanns_b200 import builder
    need_file = (args.impl == "reference") or (rank == 0 and world == 1 and not args.no_cpu_baseline)
    t1 = time.time()
    sd = builder.build_index(base, cent, lab, seed=cfg["seed"], device=dev, keep_bits=need_file)
    log(f"[bench] index build {time.time() - t1:.1f}s")
    gt_ids, gt_d = ground_truth(base, q, k)
    q_np = q.cpu().numpy()

    index_path = None
    if need_file:
        t2 = time.time()
        index_path = Path(tempfile.gettempdir()) / f"cora_bench_{args.config}.index"
        builder.write_index_file(index_path, sd, sd["bits"])
        del sd["bits"]
        log(f"[bench] index file {index_path.stat().st_size / 1e9:.2f} GB in {time.time() - t2:.1f}s")

    if args.impl == "reference":
        # the reference's own operating point: the smallest nprobe of the sweep whose
        # recall@10 on a 1000-query sample reaches the target (the rule the GPU arm uses)
        nprobe = args.nprobe
        if not nprobe:
            import py_oracle as po
            ivf = po.RefIVF(index_path) if po.ref_available() else po.oracle_from_file(index_path)
            ms = min(1000, len(q_np))
            for npb in cfg["nprobes"]:
                ids = ivf.search(q_np[:ms], k, npb, threads=os.cpu_count())
                ids = ids[1] if isinstance(ids, tuple) else ids
                nprobe = npb
                if recall_at_k(base, q[:ms], gt_ids[:ms], gt_d[:ms], ids, k) >= TARGET_RECALL:
                    break
        base_info, run = cpu_reference_qps(index_path, q_np, k, nprobe, target_seconds=4.0)
        m = int(base_info["sample"].split()[0])
        for _ in range(args.warmup):
            run(q_np[:m])
        t = time.perf_counter()
        for _ in range(args.steps):
            run(q_np[:m])
        dt = (time.perf_counter() - t) / args.steps
        v = m / dt
        rec = recall_at_k(base[:], q[:m], gt_ids[:m], gt_d[:m], run(q_np[:m]), k)
        line = dict(metric="QPS at recall@10>=0.95 (IVF-RaBitQ search)", value=v, unit="queries/s",
                    n_gpus=world, steps=args.steps, warmup=args.warmup, ms_per_step=dt * 1e3,
                    higher_is_better=True, scaling="strong", vs_baseline=None, dtype="u8+f32",
                    data="synthetic (seeded Gaussian mixture, BASELINE config 2 shape)",
                    impl="reference",
                    config=dict(workload=f"{args.config}: reference CPU IVF::search (rabitq_cpu loop)",
                                nprobe=nprobe, recall_at_10=rec, sample_queries=m),
                    cpu_baseline=dict(base_info, value=v),
                    e2e=dict(value=v, unit="queries/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
        emit(line)
        if world > 1:
            dist.destroy_process_group()
        return

    import coraanns_b200 as cb
    nprobes = [args.nprobe] if args.nprobe else cfg["nprobes"]
    # Multi-GPU layout: `shards` GPUs hold one copy of the index (cluster-sharded when > 1)
    # and world // shards such copies (replicas) each answer their own batch of the
    # config's queries (independent units, no collective between replicas): weak scaling
    # over replicas, the per-GPU work fixed as N grows. By default the index is sharded only
    # as far as memory requires (config 2 fits one GPU many times over, so every GPU holds a
    # full copy). Replica 0's batch is the N = 1 batch; replica r draws another batch from
    # the same mixture (the same seed on every shard of the replica) with its own ground
    # truth.
    shards = args.shards or auto_shards(sd, world, dev)
    if world % shards:
        raise SystemExit(f"--shards {shards} does not divide {world} GPUs")
    replicas = world // shards
    rep, srank = rank // shards, rank % shards
    nq = cfg["nq"]
    nq_total = nq * replicas
    if rep == 0:
        qs, gts = q, (gt_ids, gt_d)
    else:
        qs = make_queries(centres, cfg, nq, cfg["seed"] + 7919 * rep, dev)
        gts = ground_truth(base, qs, k)
    # A dedicated (non-default) stream: the engine enqueues every kernel of a search on it and
    # the timing events are recorded on it too. torch's default stream is the legacy NULL
    # stream, which the engine's non-blocking streams do not order against.
    stream = torch.cuda.Stream(dev)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_i = torch.empty((nq, k), dtype=torch.int32, device=dev)
    owner = None
    if shards > 1:
        # cluster-sharded: this rank keeps the clusters the shard plan gives it
        from coraanns_b200.shard import ShardedIndex, shard_plan
        groups = [dist.new_group(list(range(g * shards, (g + 1) * shards)))
                  for g in range(replicas)]
        six = ShardedIndex(local, group=groups[rep])
        apply_tuning(six.engine, args.tuning)
        six.load_search_data(sd)
        six.prepare_workspace(nq, k, max(nprobes))
        eng = six.engine
        owner = shard_plan(sd["sizes"], shards)

        def search_dev(nprobe):
            with torch.cuda.stream(stream):
                six.search_device(qs, k, nprobe, out_d, out_i)
    else:
        eng = cb.HybridIndex(local)
        apply_tuning(eng, args.tuning)
        eng.load_search_data(sd)
        eng.prepare_workspace(nq, k, max(nprobes))

        def search_dev(nprobe):
            eng.search_device(qs.data_ptr(), nq, k, nprobe, out_d.data_ptr(), out_i.data_ptr(),
                              stream.cuda_stream)
    torch.cuda.synchronize()

    def total(x, op=None):
        """Sum (or max) of a scalar over every rank."""
        if world == 1:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op or dist.ReduceOp.SUM)
        return float(t.item())

    # Operating point: the reference's two kernel types (its estimators, both with the
    # reference's refinement expression) are each swept over nprobe; the smallest nprobe whose
    # recall@10 reaches the target is kept for each, and the faster of the qualifying
    # (estimator, nprobe) configurations is the one timed below. The full-code refinement (an
    # opt-in whose distances are not the reference's) is reported beside them, not eligible.
    def recall_now():
        torch.cuda.synchronize()
        eng.check_device()
        r = recall_at_k(base, qs, gts[0], gts[1], out_i.cpu().numpy().view(np.uint32), k)
        # every shard of a replica holds the same result: count each replica once
        return total(r * nq if srank == 0 else 0.0) / nq_total

    def quick_ms(npb, reps=20):
        search_dev(npb)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        e0.record(stream)
        for _ in range(reps):
            search_dev(npb)
        e1.record(stream)
        torch.cuda.synchronize()
        return total(e0.elapsed_time(e1) / reps, dist.ReduceOp.MAX if world > 1 else None)

    estimators = {"bitwise": cb.KernelType.Bitwise, "lut": cb.KernelType.Lut4Bit}
    if args.estimator != "auto":
        estimators = {args.estimator: estimators[args.estimator]}
    sweeps, candidates = {}, {}
    for name, kt in estimators.items():
        eng.set_ip_kernel_type(kt)
        sweeps[name] = {}
        for npb in nprobes:
            search_dev(npb)
            r = recall_now()
            sweeps[name][npb] = round(r, 4)
            if r >= TARGET_RECALL:
                candidates[name] = dict(nprobe=npb, recall=round(r, 4), ms=quick_ms(npb))
                break
    eng.set_ip_kernel_type(cb.KernelType.Bitwise)
    eng.set_refine_full_code(True)
    full_code = {}
    for npb in (nprobes if args.estimator == "auto" else []):
        search_dev(npb)
        r = recall_now()
        if r >= TARGET_RECALL or npb == nprobes[-1]:
            full_code = dict(nprobe=npb, recall=round(r, 4), ms=quick_ms(npb),
                             note="opt-in full-code refinement (not the reference's distances); "
                                  "integer estimator")
            break
    eng.set_refine_full_code(False)
    if candidates:
        estimator = min(candidates, key=lambda n: candidates[n]["ms"])
        chosen = candidates[estimator]["nprobe"]
    else:  # no configuration reaches the target: the first estimator at the largest nprobe
        estimator, chosen = next(iter(estimators)), nprobes[-1]
    eng.set_ip_kernel_type(estimators[estimator])
    sweep = sweeps[estimator]
    log(f"[bench] recall sweeps {sweeps} -> {estimator} estimator, nprobe {chosen}")

    # algorithmic bytes (per-query accounting, n_c * (D/8 + 12) per probed (query, cluster)):
    # of the lows pass (the vanguard probes, ranks < vanguard), and of the whole scan
    search_dev(chosen)
    torch.cuda.synchronize()
    eng.check_device()
    probes = eng.debug("probe_ids", nq, chosen)
    local_refined = eng.get_last_submitted_count()
    cand_per_query = total(local_refined) / nq_total
    sizes = sd["sizes"].astype(np.int64)
    if owner is not None:  # this rank scans only the clusters it owns
        sizes = np.where(owner == srank, sizes, 0)
    D = int(sd["D"])
    veff = min(max(eng.get_vanguard_size(), 1), chosen)
    lows_bytes = int(sizes[probes[:, :veff]].sum()) * (D // 8 + 12)
    scan_bytes = int(sizes[probes].sum()) * (D // 8 + 12)

    # ---- timed region (device-resident queries; a single-GPU search replays its CUDA graph).
    # One repeat = K steps between CUDA events on the search stream, bracketed by a barrier
    # and device synchronisation; repeats continue until they span >= 1 s (so the clock
    # sampler sees the load), every rank running the count rank 0 chose. ms_per_step is the
    # median over repeats of the slowest rank's time per step.
    for _ in range(args.warmup):
        search_dev(chosen)
    eng.check_device()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_repeat():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            search_dev(chosen)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / args.steps

    with ClockSampler(local) as clk:
        per_step = [timed_repeat()]
        want = int(1000.0 * args.min_seconds / max(per_step[0] * args.steps, 1e-3)) + 1
        n_rep = torch.tensor([1 if args.min_seconds <= 0 else max(3, min(200, want))],
                             dtype=torch.int64, device=dev)
        if world > 1:
            dist.broadcast(n_rep, 0)
        for _ in range(int(n_rep.item()) - 1):
            per_step.append(timed_repeat())
    eng.check_device()
    rep_ms = torch.tensor(per_step, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(rep_ms, op=dist.ReduceOp.MAX)
    rep_ms = rep_ms.cpu().numpy()
    ms = float(np.median(rep_ms))
    qps = nq_total / (ms / 1e3)  # every replica's batch, answered side by side

    # ---- stage times: the same searches again with stage events (kernels launched one by
    # one), for the per-stage breakdown and the dominant kernel's duration
    eng.set_profiling(True)
    search_dev(chosen)
    eng.check_device()
    eng.stage_reset()
    for _ in range(args.steps):
        search_dev(chosen)
    torch.cuda.synchronize()
    eng.check_device()
    count, stage_tot = eng.stage_totals()
    stage_avg = {s: v / max(count, 1) for s, v in stage_tot.items()}
    eng.set_profiling(False)

    # ---- e2e through the public host API (pinned host queries, results to host) ----
    qh = torch.empty((nq, cfg["dim"]), dtype=torch.float32, pin_memory=True)
    qh.copy_(qs.cpu())
    qh_np = qh.numpy()
    if shards > 1:
        host_search = lambda: six.search(qh_np, k, chosen)  # noqa: E731
    else:
        # results land in pinned host buffers (the C ABI writes caller-provided buffers)
        od = torch.empty((nq, k), dtype=torch.float32, pin_memory=True).numpy()
        oi = torch.empty((nq, k), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
        eng.reset_buffer(qh_np)
        host_search = lambda: eng.search(qh_np, k, chosen, out=(od, oi))  # noqa: E731
    for _ in range(args.warmup):
        host_search()
    if world > 1:
        dist.barrier()
    e2e_steps = args.steps * len(rep_ms)  # about as long as the device-timed region
    t = time.perf_counter()
    for _ in range(e2e_steps):
        host_search()
    e2e_s = total((time.perf_counter() - t) / e2e_steps,
                  dist.ReduceOp.MAX if world > 1 else None)
    e2e_qps = nq_total / e2e_s

    peak, peak_src = measured_peaks()
    mode = eng.get_vanguard_mode()
    # The dominant kernel is the scan's lows pass (scan_kernel over the vanguard pairs, every
    # (pair, vector) evaluated); the main pass over the other probes skips the chunks whose
    # factor range proves them above T1 and is a few percent of the search. In rescan mode
    # (lows above budget) both passes evaluate every probed pair.
    if mode == 1:
        kern_ms, kern_bytes = stage_avg["vanguard_scan"], lows_bytes
        kern = "scan_kernel lows pass (vanguard pairs)"
    else:
        kern_ms = stage_avg["vanguard_scan"] + stage_avg["main_scan"]
        kern_bytes, kern = scan_bytes, "scan_kernel (vanguard rescan + main pass)"
    achieved = kern_bytes / (kern_ms / 1e3) / 1e9 if kern_ms > 0 else None
    traffic = profiled_traffic(args.config, estimator) if (world == 1 and mode == 1) else None
    # whole search, per-query accounting: (B_scan + B_refine) over this GPU's search time,
    # B_refine = refined survivors x (7D/8 + 8 + 4) bytes
    b_search = scan_bytes + local_refined * (7 * D // 8 + 12)
    b_query = b_search / nq
    search_gbs = b_search / (ms / 1e3) / 1e9
    roofline = dict(bound="hbm", kernel=kern, achieved=achieved,
                    peak=peak, unit="GB/s", frac=(achieved / peak) if achieved else None,
                    traffic=traffic, peak_source=peak_src,
                    algorithmic_bytes_per_launch=kern_bytes, launch_ms=kern_ms,
                    search_per_query=dict(bytes_per_query=b_query, achieved=search_gbs,
                                          frac=search_gbs / peak),
                    note="bytes = n_c*(D/8+12) per (query, probed cluster) of the launch "
                         "(per-query accounting of codes touched; cross-query reuse lets this "
                         "exceed the physical DRAM traffic, which the scan kernel keeps at a "
                         "fraction of it: it is bound by its integer dot-product pipe); "
                         "search_per_query = (B_scan + B_refine) x QPS; rank 0's launches")
    per_search = launches_per_search(chosen, k, mode, shards, estimator, metric=0)
    launches = per_search * args.steps * len(rep_ms)

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and index_path is not None:
        cpu_base, _ = cpu_reference_qps(index_path, q_np, k, chosen, target_seconds=15.0)

    sharded = None
    if world > 1 and shards == 1 and not args.no_sharded:
        # a side measurement: its failure is recorded, not fatal to the headline line (a rank
        # stuck in a collective leaves it when the process group's timeout expires)
        try:
            sharded = measure_sharded(args, sd, q, k, chosen, estimators[estimator], eng,
                                      local, world, dev, total)
        except Exception as ex:  # noqa: BLE001
            sharded = {"error": f"{type(ex).__name__}: {ex}"[:500]}

    if world == 1:
        parallelism = "single"
    elif shards == 1:
        parallelism = (f"query-parallel x{replicas} (each GPU holds the whole index and answers "
                       f"its own batch of {nq} queries; no collective on the data path)")
    else:
        parallelism = (f"{replicas} replica(s) x {shards} cluster shards, {nq} queries per "
                       f"replica (NCCL all-gather of seed and top-k keys within each replica)")
    # weak over replicas (each answers its own batch); strong when one replica is sharded
    scaling = "strong" if (replicas == 1 and world > 1) else "weak"
    if rank == 0:
        line = dict(
            metric="QPS at recall@10>=0.95 (IVF-RaBitQ search)", value=qps, unit="queries/s",
            n_gpus=world, steps=args.steps, warmup=args.warmup, ms_per_step=ms,
            higher_is_better=True, scaling=scaling, vs_baseline=None,
            dtype="i8+f32" if estimator == "bitwise" else "f16+f32",
            data="synthetic (seeded Gaussian mixture, BASELINE config 2 shape)",
            config=dict(workload=f"{args.config}: {cfg['n']} x d{cfg['dim']} L2, nlist {cfg['nlist']}, "
                                 f"8-bit RaBitQ, {nq_total} queries, topk {k}",
                        nprobe=chosen, recall_at_10=sweep.get(chosen), recall_sweep=sweep,
                        estimator=(f"{estimator} (reference KernelType::"
                                   f"{'Bitwise' if estimator == 'bitwise' else 'Lut4Bit'})"),
                        refinement="reference form: f_add_ex + g + f_rescale_ex*(128*ip1 + ip2 + kb)",
                        recall_sweeps=sweeps, qualifying=candidates,
                        full_code_refinement=full_code,
                        timed_repeats=len(rep_ms), timed_span_s=round(float(rep_ms.sum()) * args.steps / 1e3, 3),
                        ms_per_step_min_max=[float(rep_ms.min()), float(rep_ms.max())],
                        candidates_per_query=cand_per_query,
                        vanguard_mode="lows" if mode == 1 else "rescan",
                        l2_flush="inputs exceed L2 (index codes > 126 MB)",
                        stage_ms=stage_avg, shards=shards, replicas=replicas,
                        parallelism=parallelism),
            roofline=roofline, cpu_baseline=cpu_base,
            e2e=dict(value=e2e_qps, unit="queries/s", h2d_bytes_per_step=nq * cfg["dim"] * 4,
                     d2h_bytes_per_step=nq * k * 8),
            gpu_launches=launches, clocks=clk.summary())
        if sharded is not None:
            line["sharded"] = sharded
        emit(line)
    eng.close()
    if index_path is not None and index_path.exists():
        index_path.unlink()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
