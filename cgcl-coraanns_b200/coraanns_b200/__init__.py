"""Python binding of libcoraanns_b200.so (the C ABI in include/cora_b200.h).

``HybridIndex`` mirrors the reference's ``coraanns::HybridIndex``
(include/coraanns/search/hybrid.cuh:18-203 of the reference project): same method names,
argument meaning and error behaviour, with the C++ exception types mapped to
``InvalidArgument`` (std::invalid_argument, a ``LogicError``), ``LogicError``
(std::logic_error) and ``RuntimeError`` (std::runtime_error).

There is no CPU fallback: the first call into the library (creating a HybridIndex, or
``load_library()``) raises ImportError if the CUDA library was not built. The library is
mapped on that first call, not at import, so that tooling in this package that needs no GPU
engine (``coraanns_b200.builder``) can be imported without it.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "_build" / "libcoraanns_b200.so"
HEADER = PKG_ROOT.parent / "include" / "cora_b200.h"

CORA_OK, CORA_EINVAL, CORA_ESTATE, CORA_ERUNTIME, CORA_ECUDA, CORA_ENOMEM = range(6)

# Exported symbols, in the order include/cora_b200.h declares them.
EXPORTS = [
    "cora_last_error", "cora_create", "cora_destroy", "cora_load_from_raw_pointers",
    "cora_load_index_file", "cora_index_info", "cora_prepare_workspace", "cora_free_workspace",
    "cora_index_file_shard_info",
    "cora_reset_buffer", "cora_enable_exact_refine", "cora_search", "cora_search_device",
    "cora_check_device",
    "cora_seed_thresholds", "cora_capture_thresholds", "cora_set_vanguard_size",
    "cora_get_vanguard_size", "cora_set_queue_capacity", "cora_set_queue_spill_capacity",
    "cora_get_queue_capacity", "cora_set_profiling", "cora_set_candidate_stats",
    "cora_set_gpu_filter_timing", "cora_set_cross_query_reuse", "cora_set_cpu_secondary_filter",
    "cora_set_ip_kernel_type", "cora_get_ip_kernel_type", "cora_set_metric", "cora_get_metric",
    "cora_set_refine_full_code",
    "cora_get_refine_full_code", "cora_get_last_submitted_count",
    "cora_get_last_refined_count", "cora_get_last_spilled_count", "cora_get_last_gpu_filter_ms",
    "cora_debug_copy", "cora_get_last_stage_ms", "cora_stage_totals", "cora_stage_reset",
    "cora_set_vanguard_lows_budget", "cora_set_tuning", "cora_get_vanguard_mode",
    "cora_get_candidate_capacity", "cora_probe_noalloc", "cora_probe_noalloc_scratch_limit",
    "cora_probe_noalloc_status",
    "cora_load_shard_arrays",
    "cora_shard_plan", "cora_shard_configure", "cora_shard_info", "cora_shard_exchange_words",
    "cora_shard_search_begin", "cora_shard_probe_words", "cora_shard_search_probe",
    "cora_shard_search_begin_probed", "cora_shard_search_resume", "cora_shard_search_end",
]

_p = C.c_void_p
_u64 = C.c_uint64


def _sig(L, name, res, *args):
    f = getattr(L, name)
    f.restype = res
    f.argtypes = list(args)


def _bind(L):
    """Declares the C signatures on a freshly mapped library."""
    _sig(L, "cora_last_error", C.c_char_p)
    _sig(L, "cora_create", C.c_int, C.POINTER(_p), C.c_int)
    _sig(L, "cora_destroy", None, _p)
    _sig(L, "cora_load_from_raw_pointers", C.c_int, _p, _u64, _u64, _u64, _u64, _u64, _p, _p, _p, _p,
         _p, _p, _p, _p)
    _sig(L, "cora_load_index_file", C.c_int, _p, C.c_char_p)
    _sig(L, "cora_index_info", C.c_int, _p, _p)
    _sig(L, "cora_prepare_workspace", C.c_int, _p, _u64, _u64, _u64)
    _sig(L, "cora_free_workspace", None, _p)
    _sig(L, "cora_reset_buffer", C.c_int, _p, _p, _u64)
    _sig(L, "cora_enable_exact_refine", C.c_int, _p, _p, _u64, _u64, _u64, _u64)
    _sig(L, "cora_index_file_shard_info", C.c_int, C.c_char_p, C.c_uint32, C.c_uint32, _p)
    _sig(L, "cora_search", C.c_int, _p, _p, _u64, _u64, _u64, _p, _p, C.c_int)
    _sig(L, "cora_search_device", C.c_int, _p, _p, _u64, _u64, _u64, _p, _p, _p)
    _sig(L, "cora_check_device", C.c_int, _p)
    _sig(L, "cora_seed_thresholds", C.c_int, _p, _p, _u64)
    _sig(L, "cora_capture_thresholds", C.c_int, _p, _p, _u64)
    _sig(L, "cora_set_vanguard_size", C.c_int, _p, _u64)
    _sig(L, "cora_get_vanguard_size", _u64, _p)
    _sig(L, "cora_set_queue_capacity", C.c_int, _p, _u64)
    _sig(L, "cora_set_queue_spill_capacity", C.c_int, _p, _u64)
    _sig(L, "cora_get_queue_capacity", _u64, _p)
    for _n in ("cora_set_profiling", "cora_set_candidate_stats", "cora_set_gpu_filter_timing",
               "cora_set_cross_query_reuse", "cora_set_cpu_secondary_filter", "cora_set_ip_kernel_type"):
        _sig(L, _n, None, _p, C.c_int)
    _sig(L, "cora_get_ip_kernel_type", C.c_int, _p)
    _sig(L, "cora_set_metric", C.c_int, _p, C.c_int)
    _sig(L, "cora_get_metric", C.c_int, _p)
    _sig(L, "cora_set_refine_full_code", None, _p, C.c_int)
    _sig(L, "cora_get_refine_full_code", C.c_int, _p)
    _sig(L, "cora_get_last_submitted_count", _u64, _p)
    _sig(L, "cora_get_last_refined_count", _u64, _p)
    _sig(L, "cora_get_last_spilled_count", _u64, _p)
    _sig(L, "cora_get_last_gpu_filter_ms", C.c_float, _p)
    _sig(L, "cora_debug_copy", C.c_int, _p, C.c_int, _p, _u64)
    _sig(L, "cora_get_candidate_capacity", _u64, _p)
    _sig(L, "cora_get_last_stage_ms", C.c_int, _p, _p, _u64)
    _sig(L, "cora_stage_totals", C.c_int, _p, _p, _u64, _p)
    _sig(L, "cora_stage_reset", C.c_int, _p)
    _sig(L, "cora_set_vanguard_lows_budget", C.c_int, _p, _u64)
    _sig(L, "cora_get_vanguard_mode", C.c_int, _p)
    _sig(L, "cora_set_tuning", C.c_int, _p, C.c_char_p, C.c_int64)
    _sig(L, "cora_probe_noalloc", C.c_int, _p, _p, _u64, _u64, _p, _p, _p)
    _sig(L, "cora_probe_noalloc_scratch_limit", _u64)
    _sig(L, "cora_probe_noalloc_status", C.c_int, _p, _p)
    _sig(L, "cora_load_shard_arrays", C.c_int, _p, _u64, _u64, _u64, _u64, _u64, _p, _p, _p, _p,
         _p, _p, _p, _p, _p)
    _sig(L, "cora_shard_plan", C.c_int, _p, _u64, C.c_uint32, _p)
    _sig(L, "cora_shard_configure", C.c_int, _p, C.c_uint32, C.c_uint32)
    _sig(L, "cora_shard_info", C.c_int, _p, _p)
    _sig(L, "cora_shard_exchange_words", _u64, _u64, _u64)
    _sig(L, "cora_shard_search_begin", C.c_int, _p, _p, _u64, _u64, _u64, _p, _p)
    _sig(L, "cora_shard_probe_words", _u64, _u64, _u64, C.c_uint32)
    _sig(L, "cora_shard_search_probe", C.c_int, _p, _p, _u64, _u64, _u64, _p, _p)
    _sig(L, "cora_shard_search_begin_probed", C.c_int, _p, _p, _p)
    _sig(L, "cora_shard_search_resume", C.c_int, _p, _p, _p)
    _sig(L, "cora_shard_search_end", C.c_int, _p, _p, _p, _p)


_cdll = None


def load_library():
    """Maps libcoraanns_b200.so (once) and returns it; ImportError when it was not built."""
    global _cdll
    if _cdll is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
                              "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(str(LIB_PATH))
        _bind(L)
        _cdll = L
    return _cdll


class _LazyLib:
    """Forwards attribute access to the library, mapping it on first use."""

    def __getattr__(self, name):
        return getattr(load_library(), name)


_lib = _LazyLib()

STAGES = ("rotate_prep", "centroid_dist", "select_probes", "vanguard_grouping",
          "vanguard_scan", "vanguard_select", "seed_refine", "threshold", "main_grouping",
          "main_scan", "vanguard_filter", "main_refine", "merge")


class LogicError(Exception):
    """std::logic_error"""


class InvalidArgument(LogicError, ValueError):
    """std::invalid_argument (a std::logic_error in C++)"""


class CoraRuntimeError(RuntimeError):
    """std::runtime_error"""


def _check(rc):
    if rc == CORA_OK:
        return
    msg = _lib.cora_last_error().decode(errors="replace")
    if rc == CORA_EINVAL:
        raise InvalidArgument(msg)
    if rc == CORA_ESTATE:
        raise LogicError(msg)
    if rc == CORA_ENOMEM:
        raise MemoryError(msg)
    raise CoraRuntimeError(msg)


def _ptr(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def probe_noalloc_scratch_limit() -> int:
    """Bytes of the static per-device scratch block behind HybridIndex.probe_noalloc."""
    return int(_lib.cora_probe_noalloc_scratch_limit())


def index_file_shard_info(path, rank: int, world: int) -> dict:
    """The share of an index file that shard `rank` of `world` holds and reads (no GPU):
    vectors, clusters, payload bytes, and the file's total vectors."""
    out = np.zeros(4, np.uint64)
    _check(_lib.cora_index_file_shard_info(str(path).encode(), rank, world, _ptr(out)))
    return dict(vectors=int(out[0]), clusters=int(out[1]), payload_bytes=int(out[2]),
                total_vectors=int(out[3]))


class KernelType:
    Lut4Bit = 0
    Bitwise = 1


class HybridIndex:
    """coraanns::HybridIndex over the C ABI; owns one engine on one GPU."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(_lib.cora_create(C.byref(h), int(device)))
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            _lib.cora_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- loading ---------------------------------------------------------------------
    def load_from_raw_pointers(self, num_vecs, d, p_d, n_centroids, ex_b, h_centroids,
                               h_rotator, h_short_data, h_short_factors, h_long_code,
                               h_ex_factors, h_ids, h_cluster_sizes):
        arrs = [np.ascontiguousarray(a, dt) if a is not None else None for a, dt in (
            (h_centroids, np.float32), (h_rotator, np.float32), (h_short_data, np.uint32),
            (h_short_factors, np.float32), (h_long_code, np.uint8), (h_ex_factors, np.float32),
            (h_ids, np.uint32), (h_cluster_sizes, np.uint64))]
        _check(_lib.cora_load_from_raw_pointers(self._h, num_vecs, d, p_d, n_centroids, ex_b,
                                                *[_ptr(a) for a in arrs]))

    def load_search_data(self, sd: dict):
        """Load the arrays of a SearchData-layout dict (keys as oracle/py_oracle.py); its
        optional "metric" (0 L2, 1 inner product) is applied too."""
        self.set_metric(int(sd.get("metric", 0)))
        self.load_from_raw_pointers(sd["num"], sd["dim"], sd["D"], sd["nlist"], sd["ex_bits"],
                                    sd["centroids"], sd["rotator"], sd["short_data"],
                                    sd["short_factors"], sd["long_codes"], sd["ex_factors"],
                                    sd["ids"], sd["sizes"])

    def load_shard_arrays(self, sd: dict, global_sizes):
        """Load a shard from a SearchData-layout dict that holds only this shard's clusters
        (sd["sizes"]: the local sizes, zero for the other clusters; every centroid) given the
        whole index's cluster sizes; see cora_load_shard_arrays."""
        self.set_metric(int(sd.get("metric", 0)))
        arrs = [np.ascontiguousarray(sd[k], dt) for k, dt in (
            ("centroids", np.float32), ("rotator", np.float32), ("short_data", np.uint32),
            ("short_factors", np.float32), ("long_codes", np.uint8), ("ex_factors", np.float32),
            ("ids", np.uint32), ("sizes", np.uint64))]
        gs = np.ascontiguousarray(global_sizes, np.uint64)
        _check(_lib.cora_load_shard_arrays(self._h, int(sd["num"]), int(sd["dim"]), int(sd["D"]),
                                           int(sd["nlist"]), int(sd["ex_bits"]),
                                           *[_ptr(a) for a in arrs], _ptr(gs)))

    def load_index_file(self, path):
        _check(_lib.cora_load_index_file(self._h, str(path).encode()))

    def index_info(self):
        out = np.zeros(6, np.uint64)
        _check(_lib.cora_index_info(self._h, _ptr(out)))
        return dict(zip(("num", "dim", "padded_dim", "nlist", "ex_bits", "max_cluster"),
                        map(int, out)))

    # -- workspace -------------------------------------------------------------------
    def prepare_workspace(self, max_queries, max_topk, max_nprobe):
        _check(_lib.cora_prepare_workspace(self._h, max_queries, max_topk, max_nprobe))

    def free_workspace(self):
        _lib.cora_free_workspace(self._h)

    def enable_exact_refine(self, base=None, base_rows=None, base_dim=None,
                            row_stride_bytes=None, data_offset_bytes=0):
        """enable_exact_refine (hybrid.cuh:171-178). `base`: a float32 (rows, dim) array
        whose row i is the vector with original id i (its rows are copied into HBM by this
        call, or at load), or a raw pointer with the four sizes as in the C ABI; None turns
        exact refinement off."""
        if base is None:
            _check(_lib.cora_enable_exact_refine(self._h, None, 0, 0, 0, 0))
            return
        if isinstance(base, np.ndarray):
            b = np.ascontiguousarray(base, np.float32)
            self._exact_base = b  # borrowed until the rows are in HBM
            _check(_lib.cora_enable_exact_refine(self._h, _ptr(b), b.shape[0], b.shape[1],
                                                 b.shape[1] * 4, 0))
            return
        _check(_lib.cora_enable_exact_refine(self._h, C.c_void_p(base), base_rows, base_dim,
                                             row_stride_bytes, data_offset_bytes))

    def reset_buffer(self, h_queries, num_queries=None):
        q = np.ascontiguousarray(h_queries, np.float32)
        n = q.shape[0] if num_queries is None else num_queries
        _check(_lib.cora_reset_buffer(self._h, _ptr(q), n))

    # -- search ----------------------------------------------------------------------
    def search(self, h_queries, topk, nprobe, batch_q=4, num_queries=None, out=None):
        """Search host queries; results go to new arrays, or into `out` = (dists, ids), C
        arrays of shape (n, topk), float32 / uint32 (e.g. views of pinned host memory, which
        the device writes directly)."""
        q = np.ascontiguousarray(h_queries, np.float32)
        n = q.shape[0] if num_queries is None else num_queries
        if out is None:
            dists = np.empty((n, topk), np.float32)
            ids = np.empty((n, topk), np.uint32)
        else:
            dists, ids = out
            if (dists.dtype != np.float32 or ids.dtype != np.uint32
                    or dists.shape != (n, topk) or ids.shape != (n, topk)
                    or not dists.flags.c_contiguous or not ids.flags.c_contiguous):
                raise ValueError("out must be C-contiguous float32 / uint32 arrays of shape "
                                 "(num_queries, topk)")
        _check(_lib.cora_search(self._h, _ptr(q), n, topk, nprobe, _ptr(dists), _ptr(ids),
                                int(batch_q)))
        return dists, ids

    def search_device(self, d_queries: int, num_queries, topk, nprobe, d_dists: int,
                      d_ids: int, stream: int = 0):
        """Enqueue a search on device pointers (e.g. torch tensors' data_ptr())."""
        _check(_lib.cora_search_device(self._h, C.c_void_p(d_queries), num_queries, topk, nprobe,
                                       C.c_void_p(d_dists), C.c_void_p(d_ids),
                                       C.c_void_p(stream) if stream else None))

    def probe_noalloc(self, d_queries: int, num_queries, nprobe, d_probe_ids: int,
                      d_probe_dists: int, stream: int = 0):
        """Coarse probing into caller-provided device buffers; allocates nothing (static
        per-device scratch, limit probe_noalloc_scratch_limit()). Calls that overlap in
        time race on the scratch; the first call on a device must precede stream capture."""
        _check(_lib.cora_probe_noalloc(self._h, C.c_void_p(d_queries), num_queries, nprobe,
                                       C.c_void_p(d_probe_ids), C.c_void_p(d_probe_dists),
                                       C.c_void_p(stream) if stream else None))

    def probe_noalloc_status(self, stream: int = 0):
        """Synchronise and raise if the last probe_noalloc failed on the device."""
        _check(_lib.cora_probe_noalloc_status(self._h, C.c_void_p(stream) if stream else None))

    # ---- cluster sharding (see coraanns_b200.shard) ----
    def shard_configure(self, rank: int, world: int):
        _check(_lib.cora_shard_configure(self._h, rank, world))

    def shard_info(self) -> dict:
        out = np.zeros(4, np.uint64)
        _check(_lib.cora_shard_info(self._h, _ptr(out)))
        return dict(rank=int(out[0]), world=int(out[1]), vectors=int(out[2]), clusters=int(out[3]))

    def shard_search_begin(self, d_queries: int, num_queries, topk, nprobe, d_send: int,
                           stream: int = 0):
        _check(_lib.cora_shard_search_begin(self._h, C.c_void_p(d_queries), num_queries, topk,
                                            nprobe, C.c_void_p(d_send),
                                            C.c_void_p(stream) if stream else None))

    def shard_search_probe(self, d_queries: int, num_queries, topk, nprobe, d_send: int,
                           stream: int = 0):
        _check(_lib.cora_shard_search_probe(self._h, C.c_void_p(d_queries), num_queries, topk,
                                            nprobe, C.c_void_p(d_send),
                                            C.c_void_p(stream) if stream else None))

    def shard_search_begin_probed(self, d_recv: int, d_send: int):
        _check(_lib.cora_shard_search_begin_probed(self._h, C.c_void_p(d_recv),
                                                   C.c_void_p(d_send)))

    def shard_search_resume(self, d_recv: int, d_send: int):
        _check(_lib.cora_shard_search_resume(self._h, C.c_void_p(d_recv), C.c_void_p(d_send)))

    def shard_search_end(self, d_recv: int, d_dists: int, d_ids: int):
        _check(_lib.cora_shard_search_end(self._h, C.c_void_p(d_recv), C.c_void_p(d_dists),
                                          C.c_void_p(d_ids)))

    def check_device(self):
        _check(_lib.cora_check_device(self._h))

    def seed_thresholds(self, h_in, nq=None):
        t = np.ascontiguousarray(h_in, np.float32)
        _check(_lib.cora_seed_thresholds(self._h, _ptr(t), t.shape[0] if nq is None else nq))

    def capture_thresholds(self, nq):
        out = np.empty(nq, np.float32)
        _check(_lib.cora_capture_thresholds(self._h, _ptr(out), nq))
        return out

    # -- knobs -----------------------------------------------------------------------
    def set_vanguard_size(self, size):
        _check(_lib.cora_set_vanguard_size(self._h, size))

    def get_vanguard_size(self):
        return int(_lib.cora_get_vanguard_size(self._h))

    def set_queue_capacity(self, capacity):
        _check(_lib.cora_set_queue_capacity(self._h, capacity))

    def set_queue_spill_capacity(self, capacity):
        _check(_lib.cora_set_queue_spill_capacity(self._h, capacity))

    def get_queue_capacity(self):
        return int(_lib.cora_get_queue_capacity(self._h))

    def set_profiling(self, on): _lib.cora_set_profiling(self._h, int(bool(on)))
    def set_candidate_stats(self, on): _lib.cora_set_candidate_stats(self._h, int(bool(on)))
    def set_gpu_filter_timing(self, on): _lib.cora_set_gpu_filter_timing(self._h, int(bool(on)))
    def set_cross_query_reuse(self, on): _lib.cora_set_cross_query_reuse(self._h, int(bool(on)))
    def set_cpu_secondary_filter(self, on): _lib.cora_set_cpu_secondary_filter(self._h, int(bool(on)))
    def set_ip_kernel_type(self, t): _lib.cora_set_ip_kernel_type(self._h, int(t))
    def get_ip_kernel_type(self): return int(_lib.cora_get_ip_kernel_type(self._h))

    def set_metric(self, metric: int):
        """0 squared L2, 1 inner product (set from the file header by load_index_file)."""
        _check(_lib.cora_set_metric(self._h, int(metric)))

    def get_metric(self) -> int: return int(_lib.cora_get_metric(self._h))

    def set_refine_full_code(self, on):
        """Refine with <q', 128 b + u> instead of the reference's 128 ip1 + ip2 (opt-in)."""
        _lib.cora_set_refine_full_code(self._h, int(bool(on)))

    def get_refine_full_code(self): return bool(_lib.cora_get_refine_full_code(self._h))

    def get_last_submitted_count(self): return int(_lib.cora_get_last_submitted_count(self._h))
    def get_last_refined_count(self): return int(_lib.cora_get_last_refined_count(self._h))
    def get_last_spilled_count(self): return int(_lib.cora_get_last_spilled_count(self._h))
    def get_last_gpu_filter_ms(self): return float(_lib.cora_get_last_gpu_filter_ms(self._h))

    def get_last_stage_ms(self) -> dict:
        """Per-stage device milliseconds of the last search (profiling must be on)."""
        out = np.zeros(len(STAGES), np.float32)
        _check(_lib.cora_get_last_stage_ms(self._h, _ptr(out), len(STAGES)))
        return dict(zip(STAGES, map(float, out)))

    def stage_totals(self):
        """(searches summed, {stage: total ms}) since stage_reset(); profiling must be on."""
        out = np.zeros(len(STAGES), np.float64)
        cnt = np.zeros(1, np.uint64)
        _check(_lib.cora_stage_totals(self._h, _ptr(out), len(STAGES), _ptr(cnt)))
        return int(cnt[0]), dict(zip(STAGES, map(float, out)))

    def stage_reset(self):
        _check(_lib.cora_stage_reset(self._h))

    def set_vanguard_lows_budget(self, nbytes):
        _check(_lib.cora_set_vanguard_lows_budget(self._h, int(nbytes)))

    def set_tuning(self, key: str, value: int):
        _check(_lib.cora_set_tuning(self._h, key.encode(), int(value)))

    def get_vanguard_mode(self):
        """1: vanguard lower bounds kept in HBM between passes; 0: vanguard rescan."""
        return int(_lib.cora_get_vanguard_mode(self._h))

    # -- diagnostics -----------------------------------------------------------------
    def candidate_capacity(self):
        return int(_lib.cora_get_candidate_capacity(self._h))

    def debug(self, what: str, nq: int, nprobe: int = 0):
        info = self.index_info()
        D = info["padded_dim"]
        W4 = 4 * ((D + 127) // 128)
        spec = {
            "rotated": (0, np.float32, (nq, D)),
            "probe_ids": (1, np.int32, (nq, nprobe)),
            "probe_g": (2, np.float32, (nq, nprobe)),
            "cand_count": (3, np.uint32, (nq,)),
            "thresholds1": (4, np.float32, (nq,)),
            "planes": (5, np.uint32, (nq, 8, W4)),
            "scalars": (6, np.float32, (nq, 4)),
            "cand_gids": (7, np.uint32, (nq, self.candidate_capacity())),
            "approx": (8, np.float32, (nq, (info["nlist"] + 3) // 4 * 4)),
            "lut": (9, np.uint16, (nq, D // 4, 16)),
            "probe_gadd": (10, np.float32, (nq, nprobe)),
        }[what]
        out = np.empty(spec[2], spec[1])
        _check(_lib.cora_debug_copy(self._h, spec[0], _ptr(out), out.nbytes))
        return out
