"""TEST INFRASTRUCTURE ONLY — Python access to the CPU checkers.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs import
this module. It wraps:

* ``oracle/_build/libcora_oracle.so`` — the C restatement of the hybrid search path
  (contract in ``oracle/cora_oracle.h``);
* ``oracle/_ref/libcora_ref_*.so`` — the reference's own CPU code (index builder,
  ``IVF::load``/``IVF::search``, the ``SearchData`` adapter, the 7-bit ex-code inner
  product and the recall evaluator), compiled from the reference tree by
  ``oracle/Makefile``; absent on machines where that tree was never present;
* a numpy restatement of the index file reader (``ivf.hpp:403-539``) and of the
  ``SearchData`` repacking (``src/index/search_data.cpp:45-123``), pinned against the
  compiled reference adapter by the tests.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libcora_oracle.so"
REF_DIR = HERE / "_ref"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


# --------------------------------------------------------------------------------------
# Index file + SearchData restatement
# --------------------------------------------------------------------------------------
HNSW_THRESHOLD = 20000  # initializer.hpp:23


def read_ivf_file(path) -> dict:
    """Parse an IVF-RaBitQ index file (ivf.hpp:403-445 save / :447-539 load)."""
    raw = Path(path).read_bytes()
    num, dim, nlist, ex_bits = struct.unpack_from("<4Q", raw, 0)
    rot_type, metric = struct.unpack_from("<BB", raw, 32)
    off = 34
    if rot_type != 0:
        raise ValueError("only MatrixRotator (type 0) indexes are supported")
    D = (dim + 63) // 64 * 64
    sizes = np.frombuffer(raw, np.uint64, nlist, off).copy()
    off += 8 * nlist
    if int(sizes.sum()) != num:
        raise ValueError("sum of cluster sizes differs from the vector count")
    rotator = np.frombuffer(raw, np.float32, dim * D, off).reshape(dim, D).copy()
    off += 4 * dim * D
    blocks = int(((sizes + 31) // 32).sum())
    batch_bytes = blocks * (D * 4 + 32 * 12)
    ex_stride = D * ex_bits // 8 + 8 if ex_bits else 0
    payload = batch_bytes + num * ex_stride + 4 * num
    remaining = len(raw) - off
    if remaining == payload + 4 * D * nlist:
        centroids = np.frombuffer(raw, np.float32, nlist * D, off).reshape(nlist, D).copy()
        off += 4 * D * nlist
    elif remaining == payload:  # nlist >= 20000: centroids in the hnswlib sidecar
        centroids = read_hnsw_centroids(str(path) + ".hnsw", nlist, D)
    else:
        raise ValueError("index size does not match a supported centroid layout")
    batch = np.frombuffer(raw, np.uint8, batch_bytes, off)
    off += batch_bytes
    ex = np.frombuffer(raw, np.uint8, num * ex_stride, off).reshape(num, ex_stride)
    off += num * ex_stride
    ids = np.frombuffer(raw, np.uint32, num, off).copy()
    return dict(num=num, dim=dim, D=D, nlist=nlist, ex_bits=ex_bits, metric=metric,
                sizes=sizes, rotator=rotator, centroids=centroids, batch=batch, ex=ex, ids=ids)


# hnswlib's saveIndex header (third_party/.../hnswlib/hnswalg.h:685-713): offsetLevel0,
# max_elements, cur_element_count, size_data_per_element, label_offset, offsetData (u64),
# maxlevel (i32), enterpoint_node (u32), maxM, maxM0, M (u64), mult (f64),
# ef_construction (u64); then cur_element_count level-0 records of size_data_per_element
# bytes (the vector at offsetData, its u64 label at label_offset), then the upper-level
# link lists.
_HNSW_HDR = struct.Struct("<6Q iI 3Q d Q")


def read_hnsw_centroids(path, nlist, D) -> np.ndarray:
    """Rotated centroids (nlist x D) of an HNSW-initialised IVF index: element labels are
    cluster ids (initializer.hpp:207-214, :252-279)."""
    raw = Path(path).read_bytes()
    (off0, _maxel, count, per, label_off, data_off, _lvl, _ep, _mm, _mm0, _m, _mult,
     _efc) = _HNSW_HDR.unpack_from(raw, 0)
    if count != nlist or data_off + 4 * D > per or label_off + 8 > per or off0 != 0:
        raise ValueError("HNSW sidecar does not match the index's clusters")
    base = _HNSW_HDR.size
    if len(raw) < base + count * per:
        raise ValueError("truncated HNSW sidecar")
    level0 = np.frombuffer(raw, np.uint8, count * per, base).reshape(count, per)
    labels = level0[:, label_off:label_off + 8].copy().view(np.uint64).reshape(count)
    if labels.max(initial=0) >= nlist or len(np.unique(labels)) != nlist:
        raise ValueError("HNSW sidecar labels are not the cluster ids")
    cent = np.empty((nlist, D), np.float32)
    cent[labels.astype(np.int64)] = level0[:, data_off:data_off + 4 * D].copy().view(np.float32)
    return cent


_KPERM0 = [0, 8, 1, 9, 2, 10, 3, 11, 4, 12, 5, 13, 6, 14, 7, 15]
_INV_KPERM0 = [0] * 16
for _j, _p in enumerate(_KPERM0):
    _INV_KPERM0[_p] = _j


def search_data(ivf: dict) -> dict:
    """Repack as src/index/search_data.cpp:45-123 does (vectorised restatement)."""
    D, num, ex_bits = ivf["D"], ivf["num"], ivf["ex_bits"]
    W = D // 32
    sizes = ivf["sizes"].astype(np.int64)
    short = np.zeros(num * W, np.uint32)
    factors = np.zeros((num, 3), np.float32)
    rec = D * 4 + 32 * 12
    inv = np.array(_INV_KPERM0, np.int64)
    dims = np.arange(D)
    # for each (dim, v%32): byte index inside the batch and nibble shift
    byte_idx = (dims[:, None] // 8) * 32 + np.where(dims[:, None] % 8 < 4, 0, 16) + inv[np.arange(32) % 16][None, :]
    nib_hi = np.arange(32)[None, :] >= 16
    bitpos = 3 - (dims[:, None] % 8) % 4
    start, boff = 0, 0
    for c, n in enumerate(sizes):
        n = int(n)
        nb = (n + 31) // 32
        if nb:
            blk = ivf["batch"][boff:boff + nb * rec].reshape(nb, rec)
            codes = blk[:, :D * 4]                        # nb x 4D bytes
            byte = codes[:, byte_idx]                     # nb x D x 32
            nib = np.where(nib_hi[None], byte >> 4, byte & 15)
            bit = (nib >> bitpos[None]) & 1               # nb x D x 32
            bit = bit.transpose(0, 2, 1).reshape(nb * 32, D)[:n]   # n x D
            words = np.zeros((n, W), np.uint64)
            for b in range(32):
                words |= bit[:, b::32].astype(np.uint64) << np.uint64(31 - b)
            # word-major per cluster: short[start*W + w*n + v]
            short[start * W:(start + n) * W] = words.astype(np.uint32).T.reshape(-1)
            fl = blk[:, D * 4:].copy().view(np.float32).reshape(nb, 3, 32)
            factors[start:start + n] = fl.transpose(0, 2, 1).reshape(nb * 32, 3)[:n]
        start += n
        boff += nb * rec
    lc = (D * ex_bits + 7) // 8
    long_codes = np.ascontiguousarray(ivf["ex"][:, :lc])
    ex_factors = np.ascontiguousarray(ivf["ex"][:, lc:lc + 8]).view(np.float32).reshape(num, 2)
    return dict(centroids=ivf["centroids"], rotator=ivf["rotator"], short_data=short,
                short_factors=factors, long_codes=long_codes.reshape(-1).copy(),
                ex_factors=ex_factors.copy(), ids=ivf["ids"], sizes=ivf["sizes"].copy(),
                num=num, dim=ivf["dim"], D=D, nlist=ivf["nlist"], ex_bits=ex_bits,
                metric=int(ivf.get("metric", 0)))


# --------------------------------------------------------------------------------------
# C oracle
# --------------------------------------------------------------------------------------
class _Index(C.Structure):
    _fields_ = [("num", C.c_uint64), ("dim", C.c_uint64), ("padded_dim", C.c_uint64),
                ("nlist", C.c_uint64), ("ex_bits", C.c_uint64),
                ("centroids", C.c_void_p), ("rotator", C.c_void_p),
                ("short_data", C.c_void_p), ("short_factors", C.c_void_p),
                ("long_codes", C.c_void_p), ("ex_factors", C.c_void_p),
                ("ids", C.c_void_p), ("cluster_sizes", C.c_void_p),
                ("exact_base", C.c_void_p), ("exact_rows", C.c_uint64),
                ("exact_dim", C.c_uint64), ("exact_stride", C.c_uint64),
                ("refine_full_code", C.c_int), ("lut_estimator", C.c_int), ("metric", C.c_int)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle oracle`")
        L = C.CDLL(str(ORACLE_SO))
        L.cora_oracle_search.restype = C.c_int
        L.cora_oracle_search.argtypes = [C.POINTER(_Index), _f32p, C.c_uint64, C.c_uint64,
                                         C.c_uint64, C.c_uint64, C.c_void_p, _f32p, _u32p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_uint64, C.c_int]
        L.cora_oracle_search_shard.restype = C.c_int
        L.cora_oracle_search_shard.argtypes = [C.POINTER(_Index), _f32p, C.c_uint64,
                                               C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p,
                                               C.c_void_p, C.c_void_p, C.c_void_p, _f32p, _u32p,
                                               C.c_void_p, C.c_int]
        L.cora_oracle_rotate.argtypes = [C.POINTER(_Index), _f32p, C.c_uint64, _f32p]
        L.cora_oracle_query_prep.argtypes = [C.c_uint64, C.c_uint64, _f32p, C.c_uint64, _f32p,
                                             _f32p, _f32p, _f32p, _i32p, _u32p]
        L.cora_oracle_probe.argtypes = [C.POINTER(_Index), _f32p, C.c_uint64, C.c_uint64,
                                        _i32p, _f32p]
        L.cora_oracle_f32_to_f16.restype = C.c_uint16
        L.cora_oracle_f32_to_f16.argtypes = [C.c_float]
        L.cora_oracle_f16_to_f32.restype = C.c_float
        L.cora_oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.cora_oracle_query_lut.argtypes = [_f32p, C.c_uint64,
                                            np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")]
        L.cora_oracle_ip_lut.restype = C.c_float
        L.cora_oracle_ip_lut.argtypes = [_u32p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"),
                                         C.c_uint64]
        L.cora_oracle_ip_ex.restype = C.c_float
        L.cora_oracle_ip_ex.argtypes = [_f32p, _u8p, C.c_uint64]
        L.cora_oracle_ex_split.restype = C.c_float
        L.cora_oracle_ex_split.argtypes = [C.POINTER(_Index), C.c_uint64, C.c_float, C.c_float,
                                           C.c_float, C.c_float]
        L.cora_oracle_ip_total.restype = C.c_float
        L.cora_oracle_ip_total.argtypes = [_f32p, _u32p, _u8p, C.c_uint64]
        L.cora_oracle_decode_ex7.argtypes = [_u8p, C.c_uint64, _u8p]
        L.cora_oracle_ip_int.restype = C.c_int32
        L.cora_oracle_ip_int.argtypes = [C.POINTER(_Index), C.c_uint64, _u32p]
        L.cora_oracle_ip_gadd.restype = C.c_float
        L.cora_oracle_ip_gadd.argtypes = [_f32p, _f32p, C.c_uint64]
        L.cora_oracle_centroid_dist.restype = C.c_float
        L.cora_oracle_centroid_dist.argtypes = [_f32p, _f32p, C.c_uint64]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class OracleIndex:
    """Holds SearchData-layout arrays (contiguous, right dtypes) for the C oracle.
    exact_base: optional float32 (rows, dim) base vectors indexed by original id; when set,
    candidates are refined with exact squared L2 distances (HybridIndex::enable_exact_refine,
    hybrid.cuh:171-178). full_code: refine with the full 8-bit code inner product instead
    of the reference's 128 * ip1 + ip2; lut: ip1 from the fp16 LUT estimator instead of the
    integer one (cora_oracle.h)."""

    def __init__(self, sd: dict, exact_base=None, full_code=False, lut=False):
        self.sd = {
            "centroids": np.ascontiguousarray(sd["centroids"], np.float32),
            "rotator": np.ascontiguousarray(sd["rotator"], np.float32),
            "short_data": np.ascontiguousarray(sd["short_data"], np.uint32),
            "short_factors": np.ascontiguousarray(sd["short_factors"], np.float32),
            "long_codes": np.ascontiguousarray(sd["long_codes"], np.uint8),
            "ex_factors": np.ascontiguousarray(sd["ex_factors"], np.float32),
            "ids": np.ascontiguousarray(sd["ids"], np.uint32),
            "sizes": np.ascontiguousarray(sd["sizes"], np.uint64),
        }
        self.num, self.dim, self.D = int(sd["num"]), int(sd["dim"]), int(sd["D"])
        self.nlist, self.ex_bits = int(sd["nlist"]), int(sd["ex_bits"])
        s = self.sd
        self.c = _Index(self.num, self.dim, self.D, self.nlist, self.ex_bits,
                        _ptr(s["centroids"]), _ptr(s["rotator"]), _ptr(s["short_data"]),
                        _ptr(s["short_factors"]), _ptr(s["long_codes"]), _ptr(s["ex_factors"]),
                        _ptr(s["ids"]), _ptr(s["sizes"]), None, 0, 0, 0, int(bool(full_code)),
                        int(bool(lut)), int(sd.get("metric", 0)))
        self.metric = int(sd.get("metric", 0))
        self.set_exact_base(exact_base)

    @property
    def full_code(self) -> bool:
        return bool(self.c.refine_full_code)

    @full_code.setter
    def full_code(self, on):
        self.c.refine_full_code = int(bool(on))

    @property
    def lut(self) -> bool:
        return bool(self.c.lut_estimator)

    @lut.setter
    def lut(self, on):
        self.c.lut_estimator = int(bool(on))

    def query_lut(self, qr):
        """LUT estimator tables (nq, D / 4, 16) as binary16 bits (uint16)."""
        qr = np.ascontiguousarray(qr, np.float32)
        out = np.empty((qr.shape[0], self.D // 4, 16), np.uint16)
        for i in range(qr.shape[0]):
            row = np.empty(self.D * 4, np.uint16)
            lib().cora_oracle_query_lut(np.ascontiguousarray(qr[i]), self.D, row)
            out[i] = row.reshape(self.D // 4, 16)
        return out

    def set_exact_base(self, base):
        """Exact refinement against `base` (float32 (rows, dim), row = original id), or off."""
        if base is None:
            self.exact = None
            self.c.exact_base, self.c.exact_rows, self.c.exact_dim, self.c.exact_stride = \
                None, 0, 0, 0
            return
        self.exact = np.ascontiguousarray(base, np.float32)
        self.c.exact_base = _ptr(self.exact)
        self.c.exact_rows, self.c.exact_dim = self.exact.shape
        self.c.exact_stride = self.exact.shape[1]

    def search(self, q, k, nprobe, vanguard=5, thresholds=None, with_details=False,
               cand_cap=0, threads=None):
        q = np.ascontiguousarray(q, np.float32)
        nq = q.shape[0]
        dist = np.empty((nq, k), np.float32)
        ids = np.empty((nq, k), np.uint32)
        cnt = np.empty(nq, np.uint64)
        t1 = np.empty(nq, np.float32)
        pids = np.empty((nq, nprobe), np.int32)
        pg = np.empty((nq, nprobe), np.float32)
        cg = np.empty((nq, cand_cap), np.uint32) if cand_cap else None
        t0 = None if thresholds is None else np.ascontiguousarray(thresholds, np.float32)
        threads = threads or min(8, os.cpu_count() or 1)
        rc = lib().cora_oracle_search(C.byref(self.c), q, nq, k, nprobe, vanguard, _ptr(t0),
                                      dist, ids, _ptr(cnt), _ptr(t1), _ptr(pids), _ptr(pg),
                                      _ptr(cg), cand_cap, threads)
        if rc != 0:
            raise ValueError("oracle rejected the search arguments")
        if not with_details:
            return dist, ids
        return dict(dist=dist, ids=ids, cand_count=cnt, thresholds1=t1, probe_ids=pids,
                    probe_g=pg, cand_gids=cg)

    def search_shard(self, q, k, nprobe, vanguard=5, thresholds=None, thresholds1=None,
                     threads=None):
        """One shard's part of a sharded search (cora_oracle_search_shard): returns
        (seed_keys, topk_keys, dist, ids), keys as uint64 (nq, k) padded with UINT64_MAX."""
        q = np.ascontiguousarray(q, np.float32)
        nq = q.shape[0]
        seeds = np.empty((nq, k), np.uint64)
        topk = np.empty((nq, k), np.uint64)
        dist = np.empty((nq, k), np.float32)
        ids = np.empty((nq, k), np.uint32)
        t0 = None if thresholds is None else np.ascontiguousarray(thresholds, np.float32)
        t1 = None if thresholds1 is None else np.ascontiguousarray(thresholds1, np.float32)
        threads = threads or min(8, os.cpu_count() or 1)
        rc = lib().cora_oracle_search_shard(C.byref(self.c), q, nq, k, nprobe, vanguard,
                                            _ptr(t0), _ptr(t1), _ptr(seeds), _ptr(topk), dist,
                                            ids, None, threads)
        if rc != 0:
            raise ValueError("oracle rejected the search arguments")
        return seeds, topk, dist, ids

    def rotate(self, q):
        q = np.ascontiguousarray(q, np.float32)
        out = np.empty((q.shape[0], self.D), np.float32)
        lib().cora_oracle_rotate(C.byref(self.c), q, q.shape[0], out)
        return out

    def query_prep(self, qr):
        qr = np.ascontiguousarray(qr, np.float32)
        nq, D = qr.shape
        outs = [np.empty(nq, np.float32) for _ in range(4)]
        qint = np.empty((nq, D), np.int32)
        planes = np.empty((nq, 8, D // 32), np.uint32)
        lib().cora_oracle_query_prep(D, self.ex_bits, qr, nq, *outs, qint, planes)
        return dict(sumq=outs[0], k1=outs[1], kb=outs[2], width=outs[3], qint=qint, planes=planes)

    def probe(self, qr, nprobe):
        qr = np.ascontiguousarray(qr, np.float32)
        ids = np.empty((qr.shape[0], nprobe), np.int32)
        g = np.empty((qr.shape[0], nprobe), np.float32)
        lib().cora_oracle_probe(C.byref(self.c), qr, qr.shape[0], nprobe, ids, g)
        return ids, g


def oracle_from_file(path, full_code=False, lut=False) -> OracleIndex:
    return OracleIndex(search_data(read_ivf_file(path)), full_code=full_code, lut=lut)


# --------------------------------------------------------------------------------------
# Reference harness (the reference's own CPU code)
# --------------------------------------------------------------------------------------
def _cpu_has_avx512() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512bw", "avx512dq", "avx512vl"))


def ref_available() -> bool:
    return any(REF_DIR.glob("libcora_ref_*.so"))


_ref = None


def ref():
    """Load the reference harness compiled for the best ISA this host supports."""
    global _ref
    if _ref is None:
        name = "libcora_ref_avx512.so" if _cpu_has_avx512() else "libcora_ref_avx2.so"
        path = REF_DIR / name
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: the reference harness was not built")
        L = C.CDLL(str(path))
        L.ref_last_error.restype = C.c_char_p
        L.ref_build_index.restype = C.c_int
        L.ref_build_index.argtypes = [_f32p, C.c_uint64, C.c_uint64, _f32p, C.c_uint64, _u32p,
                                      C.c_int, C.c_int, C.c_int, C.c_char_p]
        L.ref_open.restype = C.c_void_p
        L.ref_open.argtypes = [C.c_char_p]
        L.ref_close.argtypes = [C.c_void_p]
        L.ref_info.argtypes = [C.c_void_p, _u64p]
        L.ref_ids.argtypes = [C.c_void_p, _u32p]
        L.ref_search_data.restype = C.c_int
        L.ref_search_data.argtypes = [C.c_char_p, _f32p, _f32p, _u32p, _f32p, _u8p, _f32p, _u64p]
        L.ref_search.restype = C.c_int
        L.ref_search.argtypes = [C.c_void_p, _f32p, C.c_uint64, C.c_uint64, C.c_uint64, _u32p,
                                 C.c_int, C.c_int]
        L.ref_ip_ex.restype = C.c_float
        L.ref_ip_ex.argtypes = [_f32p, _u8p, C.c_uint64, C.c_uint64]
        L.ref_pack_ex7.argtypes = [_u8p, _u8p, C.c_uint64]
        L.ref_recall.restype = C.c_double
        L.ref_recall.argtypes = [_f32p, C.c_uint64, C.c_uint64, _u32p, C.c_uint64, C.c_uint64,
                                 C.c_char_p, C.c_int, _u32p]
        L.ref_lib_path = str(path)
        _ref = L
    return _ref


def ref_build_index(path, data, centroids, cluster_ids, total_bits=8, metric_ip=False,
                    faster=False):
    data = np.ascontiguousarray(data, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    cids = np.ascontiguousarray(cluster_ids, np.uint32)
    rc = ref().ref_build_index(data, data.shape[0], data.shape[1], centroids,
                               centroids.shape[0], cids, total_bits, int(metric_ip),
                               int(faster), str(path).encode())
    if rc != 0:
        raise RuntimeError(ref().ref_last_error().decode())


class RefIVF:
    """The reference's IVF loaded from a file; search() is the rabitq_cpu loop."""

    def __init__(self, path):
        self.path = str(path)
        self.h = ref().ref_open(self.path.encode())
        if not self.h:
            raise RuntimeError(ref().ref_last_error().decode())
        info = np.zeros(6, np.uint64)
        ref().ref_info(self.h, info)
        self.num, self.dim, self.D, self.nlist, self.ex_bits, self.metric = map(int, info)

    def close(self):
        if getattr(self, "h", None) and _ref is not None:
            try:
                _ref.ref_close(self.h)
            except TypeError:  # interpreter shutdown
                pass
            self.h = None

    def __del__(self):
        self.close()

    def search(self, q, k, nprobe, threads=None, hacc=True):
        q = np.ascontiguousarray(q, np.float32)
        out = np.empty((q.shape[0], k), np.uint32)
        rc = ref().ref_search(self.h, q, q.shape[0], k, nprobe, out,
                              threads or os.cpu_count() or 1, int(hacc))
        if rc != 0:
            raise RuntimeError(ref().ref_last_error().decode())
        return out

    def search_data(self) -> dict:
        n, D, nl, eb = self.num, self.D, self.nlist, self.ex_bits
        lc = (D * eb + 7) // 8
        out = dict(centroids=np.empty((nl, D), np.float32),
                   rotator=np.empty((self.dim, D), np.float32),
                   short_data=np.empty(n * D // 32, np.uint32),
                   short_factors=np.empty((n, 3), np.float32),
                   long_codes=np.empty(n * lc, np.uint8),
                   ex_factors=np.empty((n, 2), np.float32),
                   sizes=np.empty(nl, np.uint64))
        rc = ref().ref_search_data(self.path.encode(), out["centroids"], out["rotator"],
                                   out["short_data"], out["short_factors"], out["long_codes"],
                                   out["ex_factors"], out["sizes"])
        if rc != 0:
            raise RuntimeError(ref().ref_last_error().decode())
        ids = np.empty(n, np.uint32)
        ref().ref_ids(self.h, ids)
        out.update(ids=ids, num=n, dim=self.dim, D=D, nlist=nl, ex_bits=eb)
        return out


# --------------------------------------------------------------------------------------
# Small numpy helpers shared by tests and the bench's CPU legs
# --------------------------------------------------------------------------------------
def _dist(b, q, metric):
    """fp64 distance of base rows b to query q: squared L2 (metric 0) or minus the inner
    product (metric 1, so that smaller is better in both)."""
    return ((b - q) ** 2).sum(-1) if metric == 0 else -(b @ q)


def exact_knn(base, queries, k, metric=0):
    """Exact top-k by (fp64 distance, id), as tools/data/generate_gt_gpu.py:114-119; for the
    inner-product metric by largest inner product."""
    b = np.asarray(base, np.float64)
    out_i = np.empty((len(queries), k), np.uint32)
    out_d = np.empty((len(queries), k), np.float64)
    for i, q in enumerate(np.asarray(queries, np.float64)):
        d = _dist(b, q, metric)
        order = np.lexsort((np.arange(len(b)), d))[:k]
        out_i[i], out_d[i] = order, d[order]
    return out_i, out_d


def distance_recall(base, queries, gt_ids, results, k, metric=0):
    """Distance-aware recall@k (recall.hpp:133-190): an id counts if it is in the GT
    top-k or its exact fp64 score is as good as the GT k-th one's (squared L2 <=, inner
    product >=); duplicates count once."""
    b = np.asarray(base, np.float64)
    hits = 0
    for i, q in enumerate(np.asarray(queries, np.float64)):
        truth = set(int(x) for x in gt_ids[i, :k])
        kth = _dist(b[int(gt_ids[i, k - 1])], q, metric)
        seen = set()
        for x in results[i, :k]:
            x = int(x)
            if x in seen or x >= len(b):
                continue
            seen.add(x)
            if x in truth or _dist(b[x], q, metric) <= kth:
                hits += 1
    return hits / (len(queries) * k)


# --------------------------------------------------------------------------------------
# Cluster-sharded search on the CPU: one shard's oracle behind the begin / resume / end
# protocol of coraanns_b200.shard.run_sharded_search, exchanging through torch CPU tensors
# (gloo). The threshold and merge steps restate gather_threshold_kernel and
# gather_merge_kernel in numpy.
# --------------------------------------------------------------------------------------
_KEY_MAX = np.uint64(0xFFFFFFFFFFFFFFFF)


def unord_f32(o):
    """Inverse of the key's order-preserving float map (ord_f32)."""
    o = np.asarray(o, np.uint32)
    u = np.where(o & np.uint32(0x80000000), o & np.uint32(0x7FFFFFFF), ~o).astype(np.uint32)
    return u.view(np.float32)


def smallest_keys_per_query(recv, world, nq, k):
    """(nq, k) smallest keys of every shard's block in an all-gathered buffer."""
    stride = nq * k + 1
    blocks = np.asarray(recv).view(np.uint64).reshape(world, stride)[:, :nq * k]
    allk = blocks.reshape(world, nq, k).transpose(1, 0, 2).reshape(nq, world * k)
    return np.sort(allk, axis=1)[:, :k]


class OracleShard:
    def __init__(self, sd_shard: dict, world: int, vanguard=5, thresholds=None, threads=None,
                 full_code=False, lut=False):
        self.o = OracleIndex(sd_shard, full_code=full_code, lut=lut)
        self.world, self.vanguard, self.T0, self.threads = world, vanguard, thresholds, threads

    def buffers(self, nq, k):
        import torch
        w = nq * k + 1
        return torch.zeros(w, dtype=torch.int64), torch.zeros(self.world * w, dtype=torch.int64)

    def begin(self, q, nq, k, nprobe, send):
        self.args = (np.asarray(q, np.float32), nq, k, nprobe)
        seeds, _, _, _ = self.o.search_shard(self.args[0], k, nprobe, self.vanguard, self.T0,
                                             threads=self.threads)
        send.numpy().view(np.uint64)[:nq * k] = seeds.ravel()

    def resume(self, recv, send):
        q, nq, k, nprobe = self.args
        kth = smallest_keys_per_query(recv.numpy(), self.world, nq, k)[:, k - 1]
        T0 = np.full(nq, np.finfo(np.float32).max, np.float32) if self.T0 is None else \
            np.asarray(self.T0, np.float32)
        T1 = np.where(kth == _KEY_MAX, T0,
                      np.minimum(T0, unord_f32((kth >> np.uint64(32)).astype(np.uint32))))
        self.T1 = T1.astype(np.float32)
        _, topk, _, _ = self.o.search_shard(q, k, nprobe, self.vanguard, self.T0, self.T1,
                                            threads=self.threads)
        buf = send.numpy().view(np.uint64)
        buf[:nq * k] = topk.ravel()
        buf[nq * k] = 0

    def end(self, recv, out_d, out_i):
        _, nq, k, _ = self.args
        keys = smallest_keys_per_query(recv.numpy(), self.world, nq, k)
        ok = keys != _KEY_MAX
        out_d[...] = np.where(ok, unord_f32((keys >> np.uint64(32)).astype(np.uint32)),
                              np.finfo(np.float32).max)
        out_i[...] = np.where(ok, (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32), 0)
