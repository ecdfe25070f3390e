"""Seeded synthetic stand-ins for the large BASELINE configurations, streamed chunk by chunk.

Tooling for bench.py and the full-size GPU tests, not the search path. The public datasets
the reference measures on (LAION / Wiki / Deep) are not available here; these generators
give vectors of the same shapes and value distributions as the BASELINE configurations:
a Gaussian mixture (centres N(0, 1), per-component sigma), optionally unit-normalised (the
inner-product configurations), with uniform or Zipf(s) component weights.

Everything is generated on the GPU from counter-based seeds: chunk j of the base comes from
its own generator seeded with (seed, j), so a chunk (or a shard) regenerates its vectors
without the others, and a 88M x 768 base (270 GB in fp32) never has to exist in memory:

* ``build_index_stream`` builds the index in two passes over the chunks (nearest-centroid
  assignment, then quantisation into the reference adapter's cluster-ordered layout, via
  ``builder``'s quantizer), writing its arrays into host memory;
* ``ground_truth_stream`` computes the exact top-k (fp32 filter, fp64 rescoring of the kept
  candidates, ties by id) in one pass;
* ``exact_scores`` computes exact fp64 scores of given (query, id) pairs in one pass, for the
  distance-aware recall of search results.
"""
from __future__ import annotations

import numpy as np
import torch

from . import builder

CHUNK = 1 << 20


class Mixture:
    """n vectors of dimension dim from a mixture of `ncomp` Gaussian components."""

    def __init__(self, n, dim, ncomp, sigma, seed, normalise=False, zipf_s=None, device="cuda",
                 chunk=CHUNK):
        self.n, self.dim, self.ncomp, self.sigma = n, dim, ncomp, sigma
        self.seed, self.normalise, self.chunk = seed, normalise, chunk
        self.dev = torch.device(device)
        g = torch.Generator(device=self.dev).manual_seed(seed)
        self.centres = torch.randn(ncomp, dim, generator=g, device=self.dev)
        if zipf_s:
            w = 1.0 / torch.arange(1, ncomp + 1, device=self.dev, dtype=torch.float64) ** zipf_s
            self.weights = (w / w.sum()).float()
        else:
            self.weights = None

    @property
    def n_chunks(self):
        return (self.n + self.chunk - 1) // self.chunk

    def _labels(self, m, g):
        if self.weights is None:
            return torch.randint(0, self.ncomp, (m,), generator=g, device=self.dev)
        return torch.multinomial(self.weights, m, replacement=True, generator=g)

    def chunk_at(self, j):
        """(vectors, component labels, first id) of chunk j; ids are consecutive."""
        s = j * self.chunk
        m = min(self.chunk, self.n - s)
        g = torch.Generator(device=self.dev).manual_seed(self.seed * 1_000_003 + 7919 * (j + 1))
        lab = self._labels(m, g)
        x = self.centres[lab] + self.sigma * torch.randn(m, self.dim, generator=g, device=self.dev)
        if self.normalise:
            x = x / x.norm(dim=1, keepdim=True)
        return x, lab, s

    def queries(self, nq, qnoise, salt=1):
        g = torch.Generator(device=self.dev).manual_seed(self.seed * 1_000_003 - salt)
        lab = self._labels(nq, g)
        q = (self.centres[lab] + self.sigma * torch.randn(nq, self.dim, generator=g, device=self.dev)
             + qnoise * torch.randn(nq, self.dim, generator=g, device=self.dev))
        if self.normalise:
            q = q / q.norm(dim=1, keepdim=True)
        return q.contiguous()


def _nearest(x, cent, cn):
    """Nearest centroid (squared L2) of each row, exact fp32 arithmetic (no TF32), in row
    blocks whose distance matrix stays near 2 GB."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    rows = max(1, (1 << 29) // cent.shape[0])
    try:
        return torch.cat([(cn[None, :] - 2 * x[s:s + rows] @ cent.T).argmin(1)
                          for s in range(0, x.shape[0], rows)])
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def train_centroids(mix: Mixture, nlist, sample=1 << 21, iters=2, init="centres"):
    """IVF partition: Lloyd iterations on a sample of the first chunks, as the reference's
    k-means + nearest assignment (tools/data/train_ivf.py). init="centres" starts at the
    generating centres (nlist == ncomp; their directions for unit-normalised data, where the
    components' means lie), where k-means would end near them for equal-weight mixtures;
    init="sample" starts at nlist vectors of the sample (as Faiss's k-means does), which gives
    heavy components of a skewed mixture several centroids."""
    xs, got, j = [], 0, 0
    while got < sample and j < mix.n_chunks:
        x, _, _ = mix.chunk_at(j)
        xs.append(x[:sample - got])
        got += xs[-1].shape[0]
        j += 1
    x = torch.cat(xs)
    if init == "sample":
        g = torch.Generator(device=mix.dev).manual_seed(mix.seed + 17)
        c = x[torch.randperm(x.shape[0], generator=g, device=mix.dev)[:nlist]].clone()
    else:
        c = mix.centres[:nlist].clone()
        if mix.normalise:
            c = c / c.norm(dim=1, keepdim=True)
    for _ in range(iters):
        a = torch.cat([_nearest(x[s:s + CHUNK], c, (c * c).sum(1)) for s in range(0, len(x), CHUNK)])
        sums = torch.zeros_like(c).index_add_(0, a, x)
        cnt = torch.bincount(a, minlength=nlist).float()
        nz = cnt > 0
        c[nz] = sums[nz] / cnt[nz, None]
    return c


def build_index_stream(mix: Mixture, cent, metric=0, seed=7, log=None):
    """Index of every vector of `mix` against centroids `cent` (nlist x dim), in the
    reference adapter's layout (the dict builder.build_index returns), arrays in host memory.
    Pass 1 assigns each vector to its nearest centroid; pass 2 quantises each chunk and
    scatters its rows to their cluster-ordered positions (ids ascending within a cluster)."""
    dev = mix.dev
    n, dim = mix.n, mix.dim
    nlist = cent.shape[0]
    D = builder.padded_dim(dim)
    W = D // 32
    lc = D * 7 // 8
    cn = (cent * cent).sum(1)
    lab = torch.empty(n, dtype=torch.int64, device=dev)
    for j in range(mix.n_chunks):
        x, _, s = mix.chunk_at(j)
        for t in range(0, x.shape[0], 1 << 18):
            lab[s + t:s + t + min(1 << 18, x.shape[0] - t)] = _nearest(x[t:t + (1 << 18)], cent, cn)
    sizes = torch.bincount(lab, minlength=nlist)
    starts = torch.cumsum(sizes, 0) - sizes
    order = torch.argsort(lab, stable=True)          # cluster order, ids ascending
    dest = torch.empty_like(order)
    dest[order] = torch.arange(n, device=dev)        # position of vector i in cluster order
    del order
    if log:
        log(f"[synthetic] assigned {n} vectors; largest cluster {int(sizes.max())}")
    P = torch.as_tensor(builder.random_rotation(dim, seed), device=dev)
    crot = (cent.double() @ P.double()).float()
    t_const = builder.const_scaling_factor(D, 7, seed + 1)
    short = np.empty(n * W, np.uint32)
    fac = np.empty((n, 3), np.float32)
    lcs = np.empty((n, lc), np.uint8)
    exf = np.empty((n, 2), np.float32)
    ids = np.empty(n, np.uint32)
    sizes_d, starts_d = sizes, starts
    for j in range(mix.n_chunks):
        x, _, s = mix.chunk_at(j)
        for t in range(0, x.shape[0], 1 << 18):
            xs = x[t:t + (1 << 18)]
            m = xs.shape[0]
            gid = torch.arange(s + t, s + t + m, device=dev)
            cl = lab[gid]
            xr = (xs.double() @ P.double()).float()
            bits, f, code, ef = builder._quantize_rows(xr, crot[cl], t_const, metric=metric)
            pos = dest[gid]
            words = builder._words(bits)                         # m x W (int64)
            i_in = pos - starts_d[cl]
            base = starts_d[cl] * W + i_in
            widx = (base[:, None] + torch.arange(W, device=dev)[None, :] * sizes_d[cl][:, None])
            short[widx.cpu().numpy().ravel()] = words.cpu().numpy().astype(np.uint32).ravel()
            pn = pos.cpu().numpy()
            fac[pn] = f.cpu().numpy()
            exf[pn] = ef.cpu().numpy()
            lcs[pn] = builder._pack_ex7(code).cpu().numpy()
            ids[pn] = gid.cpu().numpy().astype(np.uint32)
        if log and (j % 16 == 15 or j == mix.n_chunks - 1):
            log(f"[synthetic] quantised {min(n, (j + 1) * mix.chunk)} / {n}")
    return dict(num=n, dim=dim, D=D, nlist=nlist, ex_bits=7, centroids=crot.cpu().numpy(),
                rotator=P.cpu().numpy(), short_data=short, short_factors=fac,
                long_codes=lcs.reshape(-1), ex_factors=exf, ids=ids,
                sizes=sizes.cpu().numpy().astype(np.uint64), t_const=t_const, metric=metric)


def _scores(q, x, metric):
    """Distances to minimise (fp32 filter): squared L2 without ||q||^2, or -<q, x>."""
    if metric == 1:
        return -(q @ x.T)
    return (x * x).sum(1)[None, :] - 2 * (q @ x.T)


def _gt_update(best_d, best_i, x, gid, q, k, metric, keep, qblock):
    """Folds the vectors x (ids gid, int64) into the running exact top-k (best_d, best_i):
    an fp32 filter keeps the `keep` best per query, whose fp64 scores decide; order by
    (fp64 distance, id)."""
    nq = q.shape[0]
    for b in range(0, nq, qblock):
        qb = q[b:b + qblock]
        sc = _scores(qb, x, metric)
        _, vi = torch.topk(sc, min(keep, x.shape[0]), dim=1, largest=False)
        xv = x[vi].double()                                   # qb x keep x dim
        if metric == 1:
            ex = -(xv * qb.double()[:, None, :]).sum(2)
        else:
            ex = ((xv - qb.double()[:, None, :]) ** 2).sum(2)
        cd = torch.cat([best_d[b:b + qblock], ex], 1)
        ci = torch.cat([best_i[b:b + qblock], gid[vi]], 1)
        # (distance, id) order: stable sort by id, then stable by distance
        o = torch.argsort(ci, dim=1, stable=True)
        cd, ci = torch.gather(cd, 1, o), torch.gather(ci, 1, o)
        o = torch.argsort(cd, dim=1, stable=True)[:, :k]
        best_d[b:b + qblock] = torch.gather(cd, 1, o)
        best_i[b:b + qblock] = torch.gather(ci, 1, o)


def _gt_init(q, k):
    nq = q.shape[0]
    return (torch.full((nq, k), float("inf"), dtype=torch.float64, device=q.device),
            torch.zeros((nq, k), dtype=torch.int64, device=q.device))


def ground_truth_stream(mix: Mixture, q, k, metric=0, keep=None, qblock=2048):
    """Exact top-k of every query over the whole base: per chunk an fp32 filter keeps the
    `keep` best per query, whose fp64 scores are computed from the chunk's vectors; the
    final top-k is by (fp64 distance, id) over all kept candidates. Returns (ids int64,
    distances fp64): squared L2, or minus the inner product."""
    keep = keep or max(2 * k, 64)
    best_d, best_i = _gt_init(q, k)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for j in range(mix.n_chunks):
            x, _, s = mix.chunk_at(j)
            gid = torch.arange(s, s + x.shape[0], device=x.device)
            _gt_update(best_d, best_i, x, gid, q, k, metric, keep, qblock)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return best_i, best_d


def exact_scores(mix: Mixture, q, ids, metric=0):
    """fp64 distance (squared L2, or minus the inner product) of every (query, id) in `ids`
    (nq x m int64, ids >= n give +inf), one pass over the chunks."""
    ids = torch.as_tensor(ids, dtype=torch.int64, device=q.device)
    out = torch.full(ids.shape, float("inf"), dtype=torch.float64, device=q.device)
    qd = q.double()
    for j in range(mix.n_chunks):
        x, _, s = mix.chunk_at(j)
        sel = (ids >= s) & (ids < s + x.shape[0])
        if not bool(sel.any()):
            continue
        qi, col = torch.nonzero(sel, as_tuple=True)
        xv = x[ids[qi, col] - s].double()
        if metric == 1:
            out[qi, col] = -(xv * qd[qi]).sum(1)
        else:
            out[qi, col] = ((xv - qd[qi]) ** 2).sum(1)
    return out


def distance_recall(gt_ids, gt_d, res_ids, res_d_exact, k):
    """Distance-aware recall@k (recall.hpp:133-190): a returned id counts once, if it is in
    the ground truth's top k or its exact distance is <= the ground truth's k-th."""
    r = torch.as_tensor(res_ids, dtype=torch.int64, device=gt_ids.device)[:, :k]
    in_gt = (r[:, :, None] == gt_ids[:, None, :k]).any(2)
    ok = in_gt | (res_d_exact[:, :k] <= gt_d[:, k - 1:k])
    srt, _ = torch.sort(torch.where(ok, r, torch.full_like(r, -1)), dim=1)
    dup = torch.zeros_like(ok)
    dup[:, 1:] = (srt[:, 1:] == srt[:, :-1]) & (srt[:, 1:] >= 0)
    hits = (srt >= 0).sum() - dup.sum()
    return float(hits) / (r.shape[0] * k)


# ------------------------------------------------------------------------------------
# Per-shard generation (the base is generated per shard from a seed)
# ------------------------------------------------------------------------------------
class ComponentShards:
    """n vectors of a Gaussian mixture with `ncomp` equally weighted components (centres
    N(0, 1), per-component sigma) whose IVF clusters are its components: cluster c holds the
    counts[c] vectors drawn from component c (multinomial counts from the seed), and its
    centroid is the component's centre. Vector ids are cluster-major: cluster c's vectors
    are base[c] .. base[c] + counts[c] - 1. Each cluster's noise comes from its own
    generator, so a shard generates exactly its own clusters' vectors, without any other
    shard's data or any exchange."""

    def __init__(self, n, dim, ncomp, sigma, seed, device="cuda"):
        self.n, self.dim, self.ncomp, self.sigma, self.seed = n, dim, ncomp, sigma, seed
        self.dev = torch.device(device)
        rng = np.random.default_rng(seed)
        self.counts = rng.multinomial(n, np.full(ncomp, 1.0 / ncomp)).astype(np.int64)
        self.base = np.concatenate([[0], np.cumsum(self.counts)[:-1]]).astype(np.int64)
        g = torch.Generator(device=self.dev).manual_seed(seed)
        self.centres = torch.randn(ncomp, dim, generator=g, device=self.dev)

    def clusters(self, cids):
        """(vectors, cluster labels, global ids) of the clusters `cids` (ascending), in
        cluster order."""
        cids = np.asarray(cids, np.int64)
        noise = []
        for c in cids:
            g = torch.Generator(device=self.dev).manual_seed(self.seed * 1_000_003 + 7919 * (int(c) + 1))
            noise.append(torch.randn(int(self.counts[c]), self.dim, generator=g, device=self.dev))
        cnt = torch.as_tensor(self.counts[cids], device=self.dev)
        c_d = torch.as_tensor(cids, device=self.dev)
        lab = torch.repeat_interleave(c_d, cnt)
        first = torch.repeat_interleave(torch.as_tensor(self.base[cids], device=self.dev), cnt)
        start = torch.repeat_interleave(torch.cumsum(cnt, 0) - cnt, cnt)
        gid = first + torch.arange(lab.shape[0], device=self.dev) - start
        x = self.centres[lab] + self.sigma * torch.cat(noise) if noise else \
            torch.empty((0, self.dim), device=self.dev)
        return x, lab, gid

    def batches(self, keep=None, rows=1 << 22):
        """clusters() of the kept clusters (all when keep is None), ascending, in batches of
        whole clusters of about `rows` vectors."""
        cids = np.arange(self.ncomp) if keep is None else np.flatnonzero(keep)
        i = 0
        while i < len(cids):
            j, m = i, 0
            while j < len(cids) and (j == i or m + self.counts[cids[j]] <= rows):
                m += int(self.counts[cids[j]])
                j += 1
            yield self.clusters(cids[i:j])
            i = j

    def queries(self, nq, qnoise, salt=1):
        g = torch.Generator(device=self.dev).manual_seed(self.seed * 1_000_003 - salt)
        lab = torch.randint(0, self.ncomp, (nq,), generator=g, device=self.dev)
        q = (self.centres[lab] + self.sigma * torch.randn(nq, self.dim, generator=g, device=self.dev)
             + qnoise * torch.randn(nq, self.dim, generator=g, device=self.dev))
        return q.contiguous()


def shard_bytes_per_vector(dim):
    """Host bytes of one vector in a shard's SearchData arrays."""
    D = builder.padded_dim(dim)
    return D // 32 * 4 + 12 + D * 7 // 8 + 8 + 4


def build_shard(mix: ComponentShards, owner, rank, metric=0, seed=7, log=None):
    """This shard's SearchData-layout arrays (host memory): every rotated centroid, the owned
    clusters' vectors quantised against their centroid in cluster order, sizes zero for the
    other clusters (what cora_load_shard_arrays takes)."""
    dev = mix.dev
    own = np.asarray(owner) == rank
    sizes = np.where(own, mix.counts, 0).astype(np.int64)
    n = int(sizes.sum())
    dim, nlist = mix.dim, mix.ncomp
    D = builder.padded_dim(dim)
    W, lc = D // 32, D * 7 // 8
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    starts_d = torch.as_tensor(starts, device=dev)
    sizes_d = torch.as_tensor(sizes, device=dev)
    base_d = torch.as_tensor(mix.base, device=dev)
    P = torch.as_tensor(builder.random_rotation(dim, seed), device=dev)
    crot = (mix.centres.double() @ P.double()).float()
    t_const = builder.const_scaling_factor(D, 7, seed + 1)
    short = np.empty(n * W, np.uint32)
    fac = np.empty((n, 3), np.float32)
    lcs = np.empty((n, lc), np.uint8)
    exf = np.empty((n, 2), np.float32)
    ids = np.empty(n, np.uint32)
    done = 0
    for bi, (x, lab, gid) in enumerate(mix.batches(own)):
        for t in range(0, x.shape[0], 1 << 18):
            xs, cl, gi = x[t:t + (1 << 18)], lab[t:t + (1 << 18)], gid[t:t + (1 << 18)]
            xr = (xs.double() @ P.double()).float()
            bits, f, code, ef = builder._quantize_rows(xr, crot[cl], t_const, metric=metric)
            i_in = gi - base_d[cl]                               # index within the cluster
            pos = starts_d[cl] + i_in                            # position in the shard
            words = builder._words(bits)                         # m x W (int64)
            widx = ((starts_d[cl] * W + i_in)[:, None]
                    + torch.arange(W, device=dev)[None, :] * sizes_d[cl][:, None])
            short[widx.cpu().numpy().ravel()] = words.cpu().numpy().astype(np.uint32).ravel()
            pn = pos.cpu().numpy()
            fac[pn] = f.cpu().numpy()
            exf[pn] = ef.cpu().numpy()
            lcs[pn] = builder._pack_ex7(code).cpu().numpy()
            ids[pn] = gi.cpu().numpy().astype(np.uint32)
        done += x.shape[0]
        if log and bi % 16 == 15:
            log(f"[synthetic] shard {rank}: quantised {done} / {n}")
    return dict(num=n, dim=dim, D=D, nlist=nlist, ex_bits=7, centroids=crot.cpu().numpy(),
                rotator=P.cpu().numpy(), short_data=short, short_factors=fac,
                long_codes=lcs.reshape(-1), ex_factors=exf, ids=ids,
                sizes=sizes.astype(np.uint64), t_const=t_const, metric=metric)


def ground_truth_shard(mix: ComponentShards, owner, rank, q, k, metric=0, keep=None,
                       qblock=1024, rows=1 << 20):
    """Exact top-k (as ground_truth_stream) over this shard's clusters only; the global
    ground truth is the (distance, id) merge of every shard's (merge_topk)."""
    keep = keep or max(2 * k, 64)
    own = np.asarray(owner) == rank
    best_d, best_i = _gt_init(q, k)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for x, _, gid in mix.batches(own, rows=rows):  # score blocks of qblock x rows
            _gt_update(best_d, best_i, x, gid, q, k, metric, keep, qblock)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return best_i, best_d


def merge_topk(ids, dists, k):
    """Top-k by (distance, id) of per-shard results concatenated along dim 1."""
    o = torch.argsort(ids, dim=1, stable=True)
    d, i = torch.gather(dists, 1, o), torch.gather(ids, 1, o)
    o = torch.argsort(d, dim=1, stable=True)[:, :k]
    return torch.gather(i, 1, o), torch.gather(d, 1, o)


def exact_scores_shard(mix: ComponentShards, owner, rank, q, ids, metric=0):
    """exact_scores over this shard's clusters: +inf for ids held by other shards (the
    elementwise minimum over shards gives every score). Only the owned clusters that hold a
    requested id are generated."""
    ids = torch.as_tensor(ids, dtype=torch.int64, device=q.device)
    out = torch.full(ids.shape, float("inf"), dtype=torch.float64, device=q.device)
    own = np.asarray(owner) == rank
    valid = (ids >= 0) & (ids < mix.n)
    cl = np.searchsorted(mix.base, ids.clamp(0, mix.n - 1).cpu().numpy(), side="right") - 1
    need = np.zeros(mix.ncomp, bool)
    need[np.unique(cl[valid.cpu().numpy()])] = True
    need &= own
    cl_d = torch.as_tensor(cl, device=q.device)
    qd = q.double()
    for x, lab, gid in mix.batches(need):
        s, e = int(gid[0]), int(gid[-1]) + 1  # the batch's clusters are consecutive ids
        sel = valid & (ids >= s) & (ids < e) & torch.as_tensor(need, device=q.device)[cl_d]
        if not bool(sel.any()):
            continue
        qi, col = torch.nonzero(sel, as_tuple=True)
        # row of id within the batch: ids of the batch's clusters are not contiguous across
        # clusters that are not consecutive, so look each id up among gid
        pos = torch.searchsorted(gid, ids[qi, col])
        hit = (pos < gid.shape[0]) & (gid[pos.clamp(max=gid.shape[0] - 1)] == ids[qi, col])
        qi, col, pos = qi[hit], col[hit], pos[hit]
        xv = x[pos].double()
        if metric == 1:
            out[qi, col] = -(xv * qd[qi]).sum(1)
        else:
            out[qi, col] = ((xv - qd[qi]) ** 2).sum(1)
    return out
