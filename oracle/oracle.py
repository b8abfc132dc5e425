"""TEST INFRASTRUCTURE: ctypes access to the two checkers.

* :class:`Oracle` -- the CPU restatement of the reference's search path
  (``gann_oracle.c``; citations there), built into ``_build/liboracle.so``.
* :class:`RefGPU` -- the reference's own kernels compiled for sm_100a
  (``_ref/libgustann_ref.so``, see ``Makefile``); needs a GPU.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module; the product path never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libgustann_ref.so")
# the reference's source tree (GANN_REFERENCE); only needed to build REF_SO
REF_SRC = os.environ.get("GANN_REFERENCE", "")

F_HOPCAP, F_STALE, F_DUPNBR, F_NAVRACE = 1, 2, 4, 8


def build(ref: bool = True) -> None:
    """Build the C oracle, and the reference library when its sources exist."""
    targets = ["oracle"]
    if ref and REF_SRC and os.path.isdir(os.path.join(REF_SRC, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REF_SRC}", *targets], check=True)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Oracle:
    """CPU restatement; ``fma_mode`` 1 = fused ``acc += d*d`` (nvcc default)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not os.path.exists(ORACLE_SO):
                build(ref=False)
            L = C.CDLL(ORACLE_SO)
            vp = C.c_void_p
            L.oracle_open.restype = vp
            L.oracle_open.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_int, C.c_int]
            L.oracle_close.argtypes = [vp]
            L.oracle_lut.argtypes = [vp, vp, C.c_int64, vp]
            L.oracle_nav.argtypes = [vp, vp, C.c_int64, vp, vp, vp]
            L.oracle_search.restype = C.c_int
            L.oracle_search.argtypes = [vp, vp, C.c_int64, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, vp, vp, C.c_int]
            L.oracle_dim.restype = C.c_int64
            L.oracle_dim.argtypes = [vp]
            L.oracle_chunks.restype = C.c_int
            L.oracle_chunks.argtypes = [vp]
            L.oracle_set_metric.argtypes = [vp, C.c_int]
            cls._lib = L
        return cls._lib

    def __init__(self, index_file: str, pq_prefix: str, nav_dir: str | None, dtype: int, fma_mode: int = 1,
                 metric: int = 0):
        L = self.lib()
        self.h = L.oracle_open(index_file.encode(), pq_prefix.encode(), (nav_dir or "").encode(), dtype, fma_mode)
        if not self.h:
            raise RuntimeError(f"oracle_open failed for {index_file}")
        L.oracle_set_metric(self.h, metric)
        self.dim = int(L.oracle_dim(self.h))
        self.m = int(L.oracle_chunks(self.h))

    def close(self):
        if self.h:
            self.lib().oracle_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _q(self, q):
        return np.ascontiguousarray(q, dtype=np.float32).reshape(-1, self.dim)

    def lut(self, q):
        q = self._q(q)
        out = np.zeros((q.shape[0], self.m, 256), np.float32)
        self.lib().oracle_lut(self.h, _p(q), q.shape[0], _p(out))
        return out

    def nav(self, q):
        q = self._q(q)
        n = q.shape[0]
        s, e, f = np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.int32)
        self.lib().oracle_nav(self.h, _p(q), n, _p(s), _p(e), _p(f))
        return s, e, f

    def search(self, q, topk: int, ef: int, entries=None, max_hops: int | None = None, threads: int | None = None):
        """Returns (nns, dist, found, hops, flags)."""
        q = self._q(q)
        n = q.shape[0]
        nns = np.zeros((n, topk), np.int32)
        dist = np.zeros((n, topk), np.float32)
        found = np.zeros(n, np.int32)
        hops = np.zeros(n, np.uint32)
        flags = np.zeros(n, np.int32)
        ent = None if entries is None else np.ascontiguousarray(entries, dtype=np.int32)
        cap = max_hops or max(1 << 14, 64 * ef)
        self.lib().oracle_search(self.h, _p(q), n, topk, ef, cap, _p(ent) if ent is not None else None,
                                 _p(nns), _p(dist), _p(found), _p(hops), _p(flags), int(threads or 0))
        return nns, dist, found, hops, flags


class RefGPU:
    """The reference's own GustANN library on the current GPU (device 0)."""

    _lib = None

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(REF_SO)

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = C.CDLL(REF_SO)
            vp = C.c_void_p
            L.ref_open.restype = vp
            L.ref_open.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_int, C.c_int]
            L.ref_search.restype = C.c_int
            L.ref_search.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp, C.POINTER(C.c_double)]
            L.ref_lut.restype = C.c_int
            L.ref_lut.argtypes = [vp, vp, C.c_int, C.c_int, vp]
            L.ref_nav.restype = C.c_int
            L.ref_nav.argtypes = [vp, vp, C.c_int, C.c_int, vp, vp]
            L.ref_close.argtypes = [vp]
            cls._lib = L
        return cls._lib

    def __init__(self, index_file: str, pq_prefix: str, nav_dir: str | None, dtype: int, dim: int,
                 use_gpu_mem: bool = True):
        self.dim = dim
        self.h = self.lib().ref_open(index_file.encode(), pq_prefix.encode(), (nav_dir or "").encode(), dtype,
                                     int(use_gpu_mem))

    def close(self):
        if self.h:
            self.lib().ref_close(self.h)
            self.h = None

    def _q(self, q):
        return np.ascontiguousarray(q, dtype=np.float32).reshape(-1, self.dim)

    def search(self, q, topk: int, ef: int):
        q = self._q(q)
        n = q.shape[0]
        nns = np.zeros((n, topk), np.int32)
        dist = np.zeros((n, topk), np.float32)
        found = np.zeros(n, np.int32)
        rt = C.c_double(0.0)
        rc = self.lib().ref_search(self.h, _p(q), n, topk, ef, _p(nns), _p(dist), _p(found), C.byref(rt))
        if rc:
            raise RuntimeError("reference search failed")
        return nns, dist, found, rt.value

    def lut(self, q, m: int):
        q = self._q(q)
        out = np.zeros((q.shape[0], m, 256), np.float32)
        if self.lib().ref_lut(self.h, _p(q), q.shape[0], self.dim, _p(out)):
            raise RuntimeError("reference LUT failed")
        return out

    def nav(self, q):
        q = self._q(q)
        s = np.zeros(q.shape[0], np.int32)
        e = np.zeros(q.shape[0], np.int32)
        if self.lib().ref_nav(self.h, _p(q), q.shape[0], self.dim, _p(s), _p(e)):
            raise RuntimeError("reference nav failed")
        return s, e
