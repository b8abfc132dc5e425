"""Python mirror of the reference's host API, over the C ABI of libgann.so.

``GustANN`` follows ``gustann::GustANN`` (``src/ssd_search.hpp:29-83``): same
method names, argument meaning and order. Errors raise :class:`GustANNError`
(a ``RuntimeError``, as ``CHECK_CUDA`` throws ``std::runtime_error`` in
``src/common_cuda.cuh:10-17``) carrying the C status code.

The library is loaded from the package directory (``_lib/libgann.so``); there
is no fallback: if it is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

from .formats import FLOAT, UINT8

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libgann.so")

PART_BLOB_BYTES = 512   # GANN_PART_BLOB_BYTES
GANN_OK, GANN_EINVAL, GANN_EIO, GANN_ENOMEM, GANN_ECUDA, GANN_ETIMEDOUT, GANN_EUNSUPPORTED, GANN_ESTATE = range(8)
STATUS_NAMES = ["OK", "EINVAL", "EIO", "ENOMEM", "ECUDA", "ETIMEDOUT", "EUNSUPPORTED", "ESTATE"]

# Every symbol include/gann.h declares.
EXPORTS = ["gann_open", "gann_open_device", "gann_search", "gann_search_device", "gann_close", "gann_last_error",
           "gann_index_info", "gann_probe_lut", "gann_probe_entry", "gann_pivot_sample", "gann_set_option",
           "gann_search_noalloc", "gann_part_export", "gann_part_attach", "gann_hop_begin", "gann_hop_requests",
           "gann_hop_step", "gann_hop_finish", "gann_hop_free", "gann_read_pages", "gann_exact_knn",
           "gann_robust_prune", "gann_sort_unique_rows"]
GANN_OPT_ADC_MODE, GANN_OPT_PIVOT_WARPS, GANN_OPT_NEIGHBOUR_CODES = 1, 2, 3
LAYOUT_AUTO, LAYOUT_SEPARATE, LAYOUT_NEIGHBOUR_CODES = 0, 1, 2
ADC_AUTO, ADC_TABLE, ADC_PIVOT, ADC_FILTERED = 0, 1, 2, 3
METRIC_L2, METRIC_IP = 0, 1


class GustANNError(RuntimeError):
    def __init__(self, code: int, msg: str):
        self.code = code
        name = STATUS_NAMES[code] if 0 <= code < len(STATUS_NAMES) else str(code)
        super().__init__(f"GANN_{name}: {msg}")


class _Config(C.Structure):
    _fields_ = [("index_file", C.c_char_p), ("pq_file_prefix", C.c_char_p), ("nav_graph_prefix", C.c_char_p),
                ("dtype", C.c_int32), ("use_gpu_mem", C.c_int32), ("device", C.c_int32),
                ("layout", C.c_int32), ("part_count", C.c_int32), ("part_index", C.c_int32),
                ("metric", C.c_int32), ("reserved", C.c_int32 * 1)]


class _Stats(C.Structure):
    _fields_ = [("run_time", C.c_double), ("total_time", C.c_double), ("hops", C.c_int64),
                ("adc_evals", C.c_int64), ("capped_queries", C.c_int64), ("bytes_touched", C.c_int64)]


class _DeviceIndex(C.Structure):
    _fields_ = [("vectors", C.c_void_p), ("vec_stride", C.c_int64), ("adjacency", C.c_void_p),
                ("adj_stride", C.c_int32), ("max_degree", C.c_int32), ("codes", C.c_void_p),
                ("code_stride", C.c_int32), ("pq_chunks", C.c_int32), ("pivots", C.c_void_p),
                ("centroid", C.c_void_p), ("chunk_offsets", C.c_void_p), ("num_points", C.c_int64),
                ("dim", C.c_int32), ("dtype", C.c_int32), ("medoid", C.c_int64), ("device", C.c_int32),
                ("metric", C.c_int32), ("reserved", C.c_int32 * 2)]


class _Info(C.Structure):
    _fields_ = [("num_points", C.c_int64), ("dim", C.c_int32), ("max_degree", C.c_int32),
                ("pq_chunks", C.c_int32), ("dtype", C.c_int32), ("medoid", C.c_int64),
                ("node_len", C.c_int32), ("nodes_per_page", C.c_int32), ("nav_points", C.c_int32),
                ("nav_start", C.c_int32), ("device_bytes", C.c_int64)]


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python -m gustann_b200.build`")
    lib = C.CDLL(LIB_PATH)
    vp, i64, i32, fp, ip = C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p
    lib.gann_open.argtypes = [C.POINTER(_Config), C.POINTER(vp)]
    lib.gann_open_device.argtypes = [C.POINTER(_DeviceIndex), C.POINTER(vp)]
    lib.gann_search.argtypes = [vp, fp, i64, i32, i32, ip, fp, ip, C.POINTER(_Stats)]
    lib.gann_search_device.argtypes = [vp, vp, i64, i32, i32, vp, vp, vp, vp, vp]
    lib.gann_close.argtypes = [vp]
    lib.gann_last_error.restype = C.c_char_p
    lib.gann_index_info.argtypes = [vp, C.POINTER(_Info)]
    lib.gann_probe_lut.argtypes = [vp, fp, i64, fp]
    lib.gann_probe_entry.argtypes = [vp, fp, i64, ip, ip]
    lib.gann_pivot_sample.argtypes = [i64, i64, C.c_uint32, ip]
    lib.gann_set_option.argtypes = [vp, i32, i64]
    lib.gann_search_noalloc.argtypes = [C.POINTER(_DeviceIndex), vp, i64, i32, i32, vp, vp, vp, vp]
    lib.gann_part_export.argtypes = [vp, vp, i64]
    lib.gann_part_attach.argtypes = [vp, i32, C.c_char_p, i64]
    lib.gann_hop_begin.argtypes = [vp, fp, i64, i32, i32, C.POINTER(vp)]
    lib.gann_hop_requests.argtypes = [vp, ip, C.POINTER(i64)]
    lib.gann_hop_step.argtypes = [vp, vp]
    lib.gann_hop_finish.argtypes = [vp, ip, fp, ip]
    lib.gann_hop_free.argtypes = [vp]
    lib.gann_read_pages.argtypes = [C.c_char_p, ip, i64, i32, vp, i32]
    lib.gann_exact_knn.argtypes = [vp, i64, i64, i32, i32, vp, i64, i64, i32, i32, vp, vp, i32, vp]
    lib.gann_robust_prune.argtypes = [vp, i64, i64, i32, i32, vp, i64, vp, vp, i32, i32, C.c_float, vp, vp, i32, vp]
    lib.gann_sort_unique_rows.argtypes = [vp, vp, i64, i32, vp, vp, i32, vp]
    for name in EXPORTS:
        if name != "gann_last_error":
            getattr(lib, name).restype = C.c_int
    return lib


lib = _load()


def _check(rc: int) -> None:
    if rc != GANN_OK:
        raise GustANNError(rc, lib.gann_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


@dataclass
class GustANNConfig:
    """``gustann::GustANNConfig`` (``src/ssd_search.hpp:18-23``)."""

    index_file: str
    pq_file_prefix: str
    nav_graph_prefix: str = ""


@dataclass
class GustANNStats:
    """``gustann::GustANNStats`` plus the counters of ``gann_stats``."""

    run_time: float = 0.0
    total_time: float = 0.0
    hops: int = 0
    adc_evals: int = 0
    capped_queries: int = 0
    bytes_touched: int = 0


class GustANN:
    """Drop-in for ``gustann::GustANN`` on one B200 (``device``). ``metric``
    (an extension; the reference is L2-only) is :data:`METRIC_L2` or
    :data:`METRIC_IP` (distances -<q, x>)."""

    def __init__(self, data_type: int = FLOAT, device: int = 0, layout: int = 0, metric: int = METRIC_L2):
        if data_type not in (UINT8, FLOAT):
            raise GustANNError(GANN_EINVAL, "data type must be UINT8 (0) or FLOAT (1)")
        self.data_type = data_type
        self.device = device
        self.layout = layout
        self.metric = metric
        self._h = None
        self.dim = 0

    # --------------------------------------------------------------- init
    def init_pure_mem(self, config: GustANNConfig, use_gpu_mem: bool, part_count: int = 0,
                      part_index: int = 0) -> None:
        """``GustANN::init_pure_mem`` (``src/ssd_search.cu:108-112``). With
        ``part_count`` > 1 the node records are split by id range and this
        handle loads range ``part_index`` (-1: every range, on this device);
        other processes' ranges are added with :meth:`attach_part`."""
        self.close()
        cfg = _Config(config.index_file.encode(), config.pq_file_prefix.encode(),
                      (config.nav_graph_prefix or "").encode(), self.data_type, int(bool(use_gpu_mem)),
                      self.device, self.layout, part_count, part_index, self.metric)
        h = C.c_void_p()
        _check(lib.gann_open(C.byref(cfg), C.byref(h)))
        self._h = h
        self.dim = self.info()["dim"]

    @classmethod
    def from_device(cls, vectors, adjacency, codes, pivots: np.ndarray, centroid: np.ndarray,
                    chunk_offsets: np.ndarray, medoid: int, max_degree: int, device: int = 0,
                    metric: int = METRIC_L2) -> "GustANN":
        """Search over caller-owned CUDA tensors (``gann_open_device``): ``vectors``
        [n, d] uint8/float32, ``adjacency`` [n, stride] int32 (-1 = empty slot),
        ``codes`` [n, code_stride] uint8. The tensors must stay alive and may be
        rewritten between searches."""
        dt = UINT8 if vectors.dtype.itemsize == 1 else FLOAT
        g = cls(dt, device, metric=metric)
        piv = np.ascontiguousarray(pivots, np.float32)
        cen = np.ascontiguousarray(centroid, np.float32)
        off = np.ascontiguousarray(chunk_offsets, np.uint32)
        d = _DeviceIndex(vectors.data_ptr(), vectors.stride(0) * vectors.element_size(), adjacency.data_ptr(),
                         adjacency.stride(0), max_degree, codes.data_ptr(), codes.stride(0), len(off) - 1,
                         _ptr(piv), _ptr(cen), _ptr(off), vectors.shape[0], vectors.shape[1], dt, medoid, device,
                         metric)
        h = C.c_void_p()
        _check(lib.gann_open_device(C.byref(d), C.byref(h)))
        g._h = h
        g.dim = int(vectors.shape[1])
        g._keep = (vectors, adjacency, codes)
        return g

    def init_bam(self, *args, **kwargs) -> None:
        raise GustANNError(GANN_EUNSUPPORTED, "init_bam: BaM search is not provided by this build")

    # ------------------------------------------------------------- search
    def search(self, qdata: np.ndarray, num_queries: int, topk: int, ef_search: int, nns: np.ndarray,
               distances: np.ndarray, found_cnt: np.ndarray, stats: GustANNStats | None = None) -> None:
        """``GustANN::search`` (``src/ssd_search.cu:114-140``): fills ``nns``,
        ``distances`` (squared L2) and ``found_cnt`` in place."""
        self._need()
        q = np.ascontiguousarray(qdata, dtype=np.float32)
        if q.size < num_queries * self.dim:
            raise GustANNError(GANN_EINVAL, "search: qdata holds fewer than num_queries rows")
        for arr, dt, n in ((nns, np.int32, num_queries * topk), (distances, np.float32, num_queries * topk),
                           (found_cnt, np.int32, num_queries)):
            if arr.dtype != dt or not arr.flags.c_contiguous or arr.size < n:
                raise GustANNError(GANN_EINVAL, "search: output arrays must be contiguous int32/float32 of the right size")
        if getattr(self, "_hybrid", None) is not None:
            import time
            t0 = time.perf_counter()
            batch = self._hybrid[0] or max(num_queries, 1)
            rounds = 0
            for lo in range(0, num_queries, batch):
                hi = min(num_queries, lo + batch)
                n_, d_, f_, r_ = self.hop_search(q.reshape(-1, self.dim)[lo:hi], topk, ef_search,
                                                 threads=self._hybrid[1])
                nns.reshape(-1, topk)[lo:hi] = n_
                distances.reshape(-1, topk)[lo:hi] = d_
                found_cnt.reshape(-1)[lo:hi] = f_
                rounds += r_
            if stats is not None:
                stats.run_time = stats.total_time = time.perf_counter() - t0
                stats.hops = rounds
            return
        st = _Stats()
        _check(lib.gann_search(self._h, _ptr(q), num_queries, topk, ef_search, _ptr(nns), _ptr(distances),
                               _ptr(found_cnt), C.byref(st)))
        if stats is not None:
            for f, _ in _Stats._fields_:
                setattr(stats, f, getattr(st, f))

    def query(self, qdata: np.ndarray, topk: int, ef_search: int, stats: GustANNStats | None = None):
        """Convenience form of :meth:`search` returning ``(nns, distances, found_cnt)``."""
        q = np.ascontiguousarray(qdata, dtype=np.float32).reshape(-1, self.dim if self.dim else qdata.shape[-1])
        nq = q.shape[0]
        nns = np.zeros((nq, topk), np.int32)
        dist = np.zeros((nq, topk), np.float32)
        found = np.zeros(nq, np.int32)
        self.search(q, nq, topk, ef_search, nns, dist, found, stats)
        return nns, dist, found

    def search_device(self, d_queries: int, num_queries: int, topk: int, ef_search: int, d_nns: int,
                      d_distances: int, d_found_cnt: int, d_hops: int = 0, stream: int = 0) -> None:
        """Device-pointer search (``gann_search_device``); pointers are ints
        (e.g. ``tensor.data_ptr()``), ``stream`` a ``cudaStream_t`` handle."""
        self._need()
        _check(lib.gann_search_device(self._h, d_queries, num_queries, topk, ef_search, d_nns, d_distances,
                                      d_found_cnt, d_hops or None, stream or None))

    # ------------------------------------------------------------- probes
    def probe_lut(self, qdata: np.ndarray) -> np.ndarray:
        self._need()
        q = np.ascontiguousarray(qdata, dtype=np.float32).reshape(-1, self.dim)
        m = self.info()["pq_chunks"]
        out = np.zeros((q.shape[0], m, 256), np.float32)
        _check(lib.gann_probe_lut(self._h, _ptr(q), q.shape[0], _ptr(out)))
        return out

    def probe_entry(self, qdata: np.ndarray):
        self._need()
        q = np.ascontiguousarray(qdata, dtype=np.float32).reshape(-1, self.dim)
        s = np.zeros(q.shape[0], np.int32)
        e = np.zeros(q.shape[0], np.int32)
        _check(lib.gann_probe_entry(self._h, _ptr(q), q.shape[0], _ptr(s), _ptr(e)))
        return s, e

    def init_hybrid(self, config: GustANNConfig, hybrid_config=None) -> None:
        """``GustANN::init_hybrid`` (``src/ssd_search.cu:81-106``): node records
        stay in the index file; :meth:`search` and :meth:`query` then run the
        host-driven hop search (:meth:`hop_search`). ``hybrid_config`` may carry
        ``mini_batch`` and ``thread_cnt`` (``HybridExecutorConfig``)."""
        self.close()
        cfg = _Config(config.index_file.encode(), config.pq_file_prefix.encode(),
                      (config.nav_graph_prefix or "").encode(), self.data_type, 2, self.device, 1, 0, 0,
                      self.metric)
        h = C.c_void_p()
        _check(lib.gann_open(C.byref(cfg), C.byref(h)))
        self._h = h
        self.dim = self.info()["dim"]
        self._index_file = config.index_file
        self._hybrid = (getattr(hybrid_config, "mini_batch", 0) or 0, getattr(hybrid_config, "thread_cnt", 0) or 0)

    def hop_search(self, queries: np.ndarray, topk: int, ef_search: int, index_file: str | None = None,
                   threads: int = 0, read_pages=None):
        """Host-driven search, one hop per round (``gann_hop_*``): between hops
        the 4 KB page of every query's requested node is read from
        ``index_file`` (``gann_read_pages``), or by ``read_pages(ids, pages)``
        when given. Returns ``(nns, distances, found_cnt, rounds)``."""
        self._need()
        q = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, self.dim)
        nq = q.shape[0]
        index_file = index_file or getattr(self, "_index_file", None)
        npp = self.info()["nodes_per_page"]
        b = C.c_void_p()
        _check(lib.gann_hop_begin(self._h, _ptr(q), nq, topk, ef_search, C.byref(b)))
        try:
            ids = np.full(nq, -1, np.int32)
            pages = np.zeros((nq, 4096), np.uint8)
            active = C.c_int64()
            rounds = 0
            while True:
                _check(lib.gann_hop_requests(b, _ptr(ids), C.byref(active)))
                if active.value == 0:
                    break
                if read_pages is not None:
                    read_pages(ids, pages)
                else:
                    _check(lib.gann_read_pages(index_file.encode(), _ptr(ids), nq, npp, _ptr(pages), threads))
                _check(lib.gann_hop_step(b, _ptr(pages)))
                rounds += 1
            nns = np.zeros((nq, topk), np.int32)
            dist = np.zeros((nq, topk), np.float32)
            found = np.zeros(nq, np.int32)
            _check(lib.gann_hop_finish(b, _ptr(nns), _ptr(dist), _ptr(found)))
        finally:
            lib.gann_hop_free(b)
        return nns, dist, found, rounds

    def export_part(self) -> bytes:
        """``gann_part_export``: an opaque blob naming this handle's record
        range for :meth:`attach_part` in another process."""
        self._need()
        buf = C.create_string_buffer(PART_BLOB_BYTES)
        _check(lib.gann_part_export(self._h, buf, PART_BLOB_BYTES))
        return buf.raw

    def attach_part(self, part: int, blob: bytes) -> None:
        """``gann_part_attach``: map record range ``part`` exported by another
        process (peer access over NVLink)."""
        self._need()
        if len(blob) < PART_BLOB_BYTES:
            raise GustANNError(GANN_EINVAL, "blob too short")
        _check(lib.gann_part_attach(self._h, part, blob, PART_BLOB_BYTES))

    def set_option(self, option: int, value: int) -> None:
        """``gann_set_option``: ADC mode (0 auto, 1 table, 2 pivot) or pivot warps."""
        self._need()
        _check(lib.gann_set_option(self._h, option, value))

    def info(self) -> dict:
        self._need()
        inf = _Info()
        _check(lib.gann_index_info(self._h, C.byref(inf)))
        return {f: getattr(inf, f) for f, _ in _Info._fields_}

    # ---------------------------------------------------------- lifetime
    def close(self) -> None:
        if self._h is not None:
            lib.gann_close(self._h)
            self._h = None
        self._hybrid = None

    def _need(self) -> None:
        if self._h is None:
            raise GustANNError(GANN_ESTATE, "GustANN used before init_pure_mem")

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def exact_knn(base, queries, k: int, metric: int = METRIC_L2, stream: int = 0):
    """Exact ``k`` nearest rows of ``base`` for every row of ``queries``
    (``gann_exact_knn``): CUDA tensors of one dtype (uint8 or float32), rows
    16-byte aligned. Returns ``(ids int32 [nq, k], dists float32 [nq, k])`` on
    the same device, ascending by (distance, id); L2 distances are squared."""
    import torch
    if base.dtype != queries.dtype or base.dtype not in (torch.uint8, torch.float32):
        raise GustANNError(GANN_EINVAL, "exact_knn: base and queries must both be uint8 or float32")
    if not (base.is_cuda and queries.is_cuda) or base.device != queries.device:
        raise GustANNError(GANN_EINVAL, "exact_knn: tensors must be on one CUDA device")
    if base.stride(1) != 1 or queries.stride(1) != 1:
        raise GustANNError(GANN_EINVAL, "exact_knn: rows must be contiguous")
    dt = UINT8 if base.dtype == torch.uint8 else FLOAT
    nq = queries.shape[0]
    ids = torch.empty((nq, k), dtype=torch.int32, device=base.device)
    dists = torch.empty((nq, k), dtype=torch.float32, device=base.device)
    es = base.element_size()
    _check(lib.gann_exact_knn(base.data_ptr(), base.shape[0], base.stride(0) * es, base.shape[1], dt,
                              queries.data_ptr(), queries.stride(0) * es, nq, k, metric, ids.data_ptr(),
                              dists.data_ptr(), base.device.index or 0, stream or None))
    return ids, dists


def robust_prune(vectors, points, cand, cand_dist, r: int, alpha: float, stream: int = 0):
    """RobustPrune of many points on the GPU (``gann_robust_prune``):
    ``vectors`` [n, d] uint8/float32 CUDA tensor (rows 16-byte aligned),
    ``points`` [b] int32, ``cand`` [b, k] int32 candidates nearest-first (-1
    empty), ``cand_dist`` [b, k] float32 squared distances to the point.
    Returns (kept [b, r] int32 nearest-first, -1 padded; their distances)."""
    import torch
    if vectors.dtype not in (torch.uint8, torch.float32) or vectors.stride(1) != 1:
        raise GustANNError(GANN_EINVAL, "robust_prune: vectors must be uint8/float32 with contiguous rows")
    dt = UINT8 if vectors.dtype == torch.uint8 else FLOAT
    pts = points.to(torch.int32).contiguous()
    ci = cand.to(torch.int32).contiguous()
    cd = cand_dist.to(torch.float32).contiguous()
    b, k = ci.shape
    out = torch.empty((b, r), dtype=torch.int32, device=vectors.device)
    outd = torch.empty((b, r), dtype=torch.float32, device=vectors.device)
    _check(lib.gann_robust_prune(vectors.data_ptr(), vectors.shape[0], vectors.stride(0) * vectors.element_size(),
                                 vectors.shape[1], dt, pts.data_ptr(), b, ci.data_ptr(), cd.data_ptr(), k, r,
                                 float(alpha), out.data_ptr(), outd.data_ptr(), vectors.device.index or 0,
                                 stream or None))
    return out, outd


def sort_unique_rows(ids, dists, stream: int = 0):
    """Rows of (id, distance) candidates sorted by (distance, id) with empty
    slots (id < 0) and repeated ids removed, -1/+inf padded
    (``gann_sort_unique_rows``). CUDA tensors [rows, k], k <= 256; returns
    (ids int32, dists float32) of the same shape."""
    import torch
    i = ids.to(torch.int32).contiguous()
    d = dists.to(torch.float32).contiguous()
    rows, k = i.shape
    oi = torch.empty_like(i)
    od = torch.empty_like(d)
    _check(lib.gann_sort_unique_rows(i.data_ptr(), d.data_ptr(), rows, k, oi.data_ptr(), od.data_ptr(),
                                     i.device.index or 0, stream or None))
    return oi, od


def pivot_sample(n: int, s: int, seed: int = 114514) -> np.ndarray:
    """Sorted pivot-graph sample ids (``bin/gen_small_file.cpp:18-40`` sampling)."""
    out = np.zeros(s, np.int32)
    _check(lib.gann_pivot_sample(n, s, seed, _ptr(out)))
    return out
