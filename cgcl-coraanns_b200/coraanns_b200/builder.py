"""IVF-RaBitQ index builder (offline tooling, not the search hot path).

A vectorised restatement of the reference's CPU quantizer in its "faster" mode
(third_party/rabitq/include/rabitqlib/quantization/rabitq_impl.hpp:76-137 one-bit codes and
factors, :379-500 ex codes with a constant rescale factor t_const, :263-333 for t_const
itself; apps/build_index.cpp's `faster` flag), running on torch tensors so the same code
builds small test indexes on the CPU and 10^7-vector bench indexes on a GPU.

Outputs the reference adapter's packed layout (src/index/search_data.cpp:45-123) that
HybridIndex.load_from_raw_pointers consumes, and can write the reference index file
(ivf.hpp:403-445) so the reference's own IVF::load / IVF::search read the same index.
Factors are computed in fp64 and rounded to fp32 once, so they can differ from the
reference builder's fp32 Eigen sums in the last bits.
"""
from __future__ import annotations

import heapq
import struct
from pathlib import Path

import numpy as np
import torch

KPERM0 = [0, 8, 1, 9, 2, 10, 3, 11, 4, 12, 5, 13, 6, 14, 7, 15]
EPS0 = 1.9  # rabitq_impl.hpp:18
TIGHT_START = [0, 0.15, 0.20, 0.52, 0.59, 0.71, 0.75, 0.77, 0.81]  # rabitq_impl.hpp:263-273


def padded_dim(dim: int) -> int:
    return (dim + 63) // 64 * 64


def random_rotation(dim: int, seed: int) -> np.ndarray:
    """MatrixRotator (utils/rotator.hpp:57-71): first `dim` rows of Q^T, Q from the QR
    decomposition of a padded_dim x padded_dim Gaussian matrix (seeded here)."""
    D = padded_dim(dim)
    g = np.random.default_rng(seed).normal(size=(D, D))
    q, _ = np.linalg.qr(g)
    return np.ascontiguousarray(q.T[:dim]).astype(np.float32)


def best_rescale_factor(o_abs: np.ndarray, ex_bits: int) -> float:
    """rabitq_impl.hpp:275-333: the t maximising <o, (code + 0.5)> / ||code + 0.5||."""
    k_eps, k_nenum = 1e-5, 10
    dim = len(o_abs)
    max_o = float(o_abs.max())
    t_end = ((1 << ex_bits) - 1 + k_nenum) / max_o
    t_start = t_end * TIGHT_START[ex_bits]
    cur = (t_start * o_abs + k_eps).astype(np.int64)
    sqr_den = dim * 0.25 + float((cur * cur + cur).sum())
    num = float(((cur + 0.5) * o_abs).sum())
    heap = [((cur[i] + 1) / o_abs[i], i) for i in range(dim) if o_abs[i] > 0]
    heapq.heapify(heap)
    max_ip, t = 0.0, 0.0
    while heap:
        cur_t, i = heapq.heappop(heap)
        cur[i] += 1
        u = int(cur[i])
        sqr_den += 2 * u
        num += float(o_abs[i])
        ip = num / np.sqrt(sqr_den)
        if ip > max_ip:
            max_ip, t = ip, cur_t
        if u < (1 << ex_bits) - 1:
            t_next = (u + 1) / o_abs[i]
            if t_next < t_end:
                heapq.heappush(heap, (t_next, i))
    return t


def const_scaling_factor(D: int, ex_bits: int = 7, seed: int = 12345, samples: int = 100) -> float:
    """rabitq_impl.hpp:362-377: mean best t over normalised |Gaussian| vectors (seeded)."""
    g = np.abs(np.random.default_rng(seed).normal(size=(samples, D)))
    g /= np.linalg.norm(g, axis=1, keepdims=True)
    return float(np.mean([best_rescale_factor(row, ex_bits) for row in g]))


def _pack_ex7(code: torch.Tensor) -> torch.Tensor:
    """packing_7bit_excode (pack_excode.hpp:216-264), per 64 dims -> 56 bytes."""
    n, D = code.shape
    c = code.view(n, D // 64, 64).to(torch.int32)
    out = torch.empty((n, D // 64, 56), dtype=torch.int32, device=code.device)
    lo6 = c[:, :, :48] & 63
    hi = c[:, :, 48:64]
    out[:, :, 0:16] = lo6[:, :, 0:16] | ((hi & 3) << 6)
    out[:, :, 16:32] = lo6[:, :, 16:32] | (((hi >> 2) & 3) << 6)
    out[:, :, 32:48] = lo6[:, :, 32:48] | (((hi >> 4) & 3) << 6)
    top = (c >> 6) & 1  # dim d -> bit 8*(d%8) + d//8 of a little-endian u64
    d = torch.arange(64, device=code.device)
    byte_idx = d % 8
    bit_in_byte = d // 8
    tb = torch.zeros((n, D // 64, 8), dtype=torch.int32, device=code.device)
    for j in range(64):
        tb[:, :, int(byte_idx[j])] |= top[:, :, j] << int(bit_in_byte[j])
    out[:, :, 48:56] = tb
    return out.to(torch.uint8).reshape(n, D // 64 * 56)


def _words(bits: torch.Tensor) -> torch.Tensor:
    """n x D bool -> n x D/32 uint32 words, dim 32w+b at bit 31-b."""
    n, D = bits.shape
    b = bits.view(n, D // 32, 32).to(torch.int64)
    w = (b << (31 - torch.arange(32, device=bits.device))).sum(2)
    return w.to(torch.int64)


def build_index(data, centroids, assign, seed: int = 7, device="cpu", chunk: int = 1 << 20,
                keep_bits: bool = False, rotator=None, rotated_centroids=None,
                t_const: float | None = None, metric: int = 0) -> dict:
    """Build an 8-bit (1 + 7 ex bits) index, metric 0 (squared L2) or 1 (inner product).
    data n x dim, centroids nlist x dim, assign n cluster ids. Returns the adapter layout
    dict (see oracle/py_oracle.py keys), plus 'bits' (n x D bool, cluster order) when
    keep_bits.

    The random pieces are seeded from `seed`; to quantise against another builder's choices
    (e.g. the reference's, which draws them unseeded) pass them in: `rotator` (dim x D),
    `rotated_centroids` (nlist x D, used as given) and `t_const` (the ex-code rescale
    constant of the "faster" mode)."""
    dev = torch.device(device)
    data = torch.as_tensor(np.asarray(data) if not torch.is_tensor(data) else data)
    n, dim = data.shape
    D = padded_dim(dim)
    nlist = int(centroids.shape[0])
    P = torch.as_tensor(np.asarray(rotator, np.float32) if rotator is not None
                        else random_rotation(dim, seed), device=dev)
    if rotated_centroids is not None:
        crot = torch.as_tensor(np.asarray(rotated_centroids, np.float32), device=dev)
    else:
        cent = torch.as_tensor(np.asarray(centroids, np.float32) if not torch.is_tensor(centroids)
                               else centroids, device=dev).float()
        crot = (cent.double() @ P.double()).float()
    if t_const is None:
        t_const = const_scaling_factor(D, 7, seed + 1)
    a = torch.as_tensor(np.asarray(assign) if not torch.is_tensor(assign) else assign,
                        device=dev).long()
    order = torch.argsort(a, stable=True)
    sizes = torch.bincount(a, minlength=nlist)
    starts = torch.cumsum(sizes, 0) - sizes
    W = D // 32
    short = torch.empty(n * W, dtype=torch.int64, device=dev)
    fac = torch.empty((n, 3), dtype=torch.float32, device=dev)
    lcs = torch.empty((n, D * 7 // 8), dtype=torch.uint8, device=dev)
    exf = torch.empty((n, 2), dtype=torch.float32, device=dev)
    all_bits = torch.empty((n, D), dtype=torch.bool, device=dev) if keep_bits else None
    a_sorted = a[order]
    pos = torch.arange(n, device=dev)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        idx = order[s:e].to(data.device)
        x = data[idx].to(dev).float()
        xr = (x.double() @ P.double()).float()
        cl = a_sorted[s:e]
        bits, f, code, ef = _quantize_rows(xr, crot[cl], t_const, metric=metric)
        fac[s:e], exf[s:e], lcs[s:e] = f, ef, _pack_ex7(code)
        if keep_bits:
            all_bits[s:e] = bits
        # word-major per cluster: short[start*W + w*n_c + i]
        words = _words(bits)                      # m x W
        i_in = pos[s:e] - starts[cl]
        base = starts[cl] * W + i_in
        for w in range(W):
            short[base + w * sizes[cl]] = words[:, w]
    out = dict(num=n, dim=dim, D=D, nlist=nlist, ex_bits=7,
               centroids=crot.cpu().numpy(), rotator=P.cpu().numpy(),
               short_data=short.to(torch.int64).cpu().numpy().astype(np.uint32),
               short_factors=fac.cpu().numpy(), long_codes=lcs.cpu().numpy().reshape(-1),
               ex_factors=exf.cpu().numpy(), ids=order.cpu().numpy().astype(np.uint32),
               sizes=sizes.cpu().numpy().astype(np.uint64), t_const=t_const, metric=metric)
    if keep_bits:
        out["bits"] = all_bits.cpu().numpy()
    return out


def _quantize_rows(xr, crows, t_const, ex_bits=7, metric=0):
    """Quantise rotated vectors xr (m x D) against their rotated centroids crows (m x D):
    one-bit code b = [r > 0] and factors (rabitq_impl.hpp:76-137), ex code with the constant
    rescale factor and its factors (rabitq_impl.hpp:379-500), for squared L2 (metric 0) or
    inner product (metric 1, the METRIC_IP branches: f_add = 1 - <r, c> + |r|^2 <c, xu> /
    <r, xu>, f_rescale = -|r|^2 / <r, xu>, f_error without the factor 2, f_rescale_ex =
    -|r| / ipnorm). Returns bits (m x D bool), factors (m x 3 f32), ex codes (m x D uint8 in
    [0, 127]) and ex factors (m x 2 f32)."""
    r = xr.double() - crows.double()
    c = crows.double()
    D = r.shape[1]
    bits = r > 0
    xu = bits.double() - 0.5
    l2_sqr = (r * r).sum(1)
    l2_norm = l2_sqr.sqrt()
    ip_resi = (r * xu).sum(1)
    ip_cent = (c * xu).sum(1)
    ip_resi = torch.where(ip_resi == 0, torch.full_like(ip_resi, float("inf")), ip_resi)
    xu_sq = (xu * xu).sum(1)
    tmp_err = l2_norm * EPS0 * torch.sqrt(((l2_sqr * xu_sq) / (ip_resi * ip_resi) - 1) / (D - 1))
    ip_rc = (r * c).sum(1)
    if metric == 1:
        fac = torch.stack([1 - ip_rc + l2_sqr * ip_cent / ip_resi, -l2_sqr / ip_resi, tmp_err],
                          1).float()
    else:
        fac = torch.stack([l2_sqr + 2 * l2_sqr * ip_cent / ip_resi, -2 * l2_sqr / ip_resi,
                           2 * tmp_err], 1).float()
    o = (r / l2_norm.clamp_min(1e-300)[:, None]).abs()
    code = torch.clamp((t_const * o + 1e-5).floor(), max=(1 << ex_bits) - 1).to(torch.int64)
    ipnorm = ((code.double() + 0.5) * o).sum(1)
    inv = (1.0 / ipnorm).float()
    inv = torch.where(torch.isfinite(inv) & (inv != 0), inv, torch.ones_like(inv)).double()
    mask = (1 << ex_bits) - 1
    code = torch.where(r < 0, (~code) & mask, code)
    total = code + ((r >= 0).to(torch.int64) << ex_bits)
    xu_ex = total.double() - ((1 << ex_bits) - 0.5)
    ip_resi_ex = (r * xu_ex).sum(1)
    ip_cent_ex = (c * xu_ex).sum(1)
    ip_resi_ex = torch.where(ip_resi_ex == 0, torch.full_like(ip_resi_ex, float("inf")), ip_resi_ex)
    if metric == 1:
        exf = torch.stack([1 - ip_rc + l2_sqr * ip_cent_ex / ip_resi_ex, inv * -l2_norm], 1).float()
    else:
        exf = torch.stack([l2_sqr + 2 * l2_sqr * ip_cent_ex / ip_resi_ex, inv * -2 * l2_norm],
                          1).float()
    return bits, fac, code.to(torch.uint8), exf


def write_index_file(path, sd: dict, bits: np.ndarray):
    """Write the reference IVF file (ivf.hpp:403-445) for an index built above. `bits` is the
    n x D bool 1-bit code matrix in cluster order (build_index(keep_bits=True)['bits'])."""
    n, dim, D, nlist = int(sd["num"]), int(sd["dim"]), int(sd["D"]), int(sd["nlist"])
    sizes = sd["sizes"].astype(np.uint64)
    with open(path, "wb") as f:
        f.write(struct.pack("<4Q", n, dim, nlist, 7))
        f.write(struct.pack("<BB", 0, int(sd.get("metric", 0))))  # matrix rotator, metric
        f.write(sizes.tobytes())
        f.write(np.ascontiguousarray(sd["rotator"], np.float32).tobytes())
        f.write(np.ascontiguousarray(sd["centroids"], np.float32).tobytes())
        # FastScan batches (fastscan.hpp:69-106) + 3 x 32 factors (data_layout.hpp:9-28)
        compact = np.packbits(bits.astype(np.uint8), axis=1, bitorder="big")  # n x D/8
        perm = np.array(KPERM0)
        start = 0
        fac = sd["short_factors"]
        for c in range(nlist):
            nc = int(sizes[c])
            for b0 in range(0, nc, 32):
                m = min(32, nc - b0)
                blk = np.zeros((32, D // 8), np.uint8)
                blk[:m] = compact[start + b0:start + b0 + m]
                hi, lo = blk >> 4, blk & 15
                out = np.empty((D // 8, 32), np.uint8)
                out[:, :16] = (hi[perm] | (hi[perm + 16] << 4)).T
                out[:, 16:] = (lo[perm] | (lo[perm + 16] << 4)).T
                f.write(out.tobytes())
                ff = np.zeros((3, 32), np.float32)
                ff[:, :m] = fac[start + b0:start + b0 + m].T
                f.write(ff.tobytes())
            start += nc
        lc = D * 7 // 8
        ex = np.empty((n, lc + 8), np.uint8)
        ex[:, :lc] = sd["long_codes"].reshape(n, lc)
        ex[:, lc:] = np.ascontiguousarray(sd["ex_factors"], np.float32).view(np.uint8).reshape(n, 8)
        f.write(ex.tobytes())
        f.write(np.ascontiguousarray(sd["ids"], np.uint32).tobytes())
