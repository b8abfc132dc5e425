"""On-disk formats read by GustANN's search path, written and read with numpy.

Every layout here is the one the reference search code parses; the library's
native loader (``csrc/gann_loader.cpp``) reads the same bytes.

* DiskANN disk index (``*_disk.index``): page 0 is a header, then 4 KB pages
  holding ``npp`` fixed-size records each. Header parse: ``src/layout.cpp:25-54``;
  record addressing ``src/impl/pure_mem.cuh:261-292``.
* PQ pivots (``<prefix>_pivots.bin``) and codes (``<prefix>_compressed.bin``):
  ``src/pq_search.cu:56-121,187-201``.
* Pivot ("nav") graph directory: ``nav_index``, ``nav_index.data``, ``map.txt``:
  ``src/nav_graph.cu:41-100``; file names ``src/ssd_search.cu:55-79``.
* Query / ground-truth vectors (fvecs, bvecs, ivecs) and ``bin`` files:
  ``bin/utils.hpp:23-88``.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

PAGE_SIZE = 4096
NUM_PIVOTS = 256
UINT8 = 0
FLOAT = 1
DTYPES = {UINT8: np.uint8, FLOAT: np.float32}


def np_dtype(dtype: int):
    if dtype not in DTYPES:
        raise ValueError(f"unknown data type {dtype}")
    return DTYPES[dtype]


# --------------------------------------------------------------------------- bin


def write_bin(path: str, arr: np.ndarray, offset: int | None = None) -> int:
    """``int32 npts, int32 ndim`` + row-major data. Returns bytes written."""
    arr = np.ascontiguousarray(arr)
    if arr.ndim == 1:
        arr = arr.reshape(-1, 1)
    npts, ndim = arr.shape
    payload = struct.pack("<ii", npts, ndim) + arr.tobytes()
    mode = "r+b" if (offset is not None and os.path.exists(path)) else "wb"
    with open(path, mode) as f:
        if offset is not None:
            f.seek(offset)
        f.write(payload)
    return len(payload)


def read_bin(path: str, dtype, offset: int = 0) -> np.ndarray:
    with open(path, "rb") as f:
        f.seek(offset)
        npts, ndim = struct.unpack("<ii", f.read(8))
        data = np.frombuffer(f.read(npts * ndim * np.dtype(dtype).itemsize), dtype=dtype)
    return data.reshape(npts, ndim)


# --------------------------------------------------------------- vecs files


def write_vecs(path: str, arr: np.ndarray) -> None:
    """fvecs / ivecs / bvecs: per row ``int32 d`` then ``d`` elements."""
    arr = np.ascontiguousarray(arr)
    n, d = arr.shape
    head = np.full((n, 1), d, dtype=np.int32).view(np.uint8)
    body = arr.view(np.uint8).reshape(n, -1)
    with open(path, "wb") as f:
        f.write(np.concatenate([head, body], axis=1).tobytes())


def read_vecs(path: str, dtype) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.uint8)
    if raw.size < 4:
        raise ValueError(f"{path}: too short")
    d = int(raw[:4].view(np.int32)[0])
    item = np.dtype(dtype).itemsize
    row = 4 + d * item
    if d <= 0 or raw.size % row:
        raise ValueError(f"{path}: bad vecs file (d={d}, size={raw.size})")
    return raw.reshape(-1, row)[:, 4:].copy().view(dtype).reshape(-1, d)


# ------------------------------------------------------------- disk index


@dataclass
class DiskLayout:
    """Header fields of a DiskANN disk index (``src/layout.hpp:8-25``)."""

    num_data: int
    num_dims: int
    medoid: int
    max_node_len: int
    nodes_per_page: int
    data_size: int          # bytes of one vector
    max_m0: int             # neighbour slots per record
    num_pages: int          # data pages (header page excluded)


def record_geometry(num_dims: int, elem: int, max_m0: int) -> tuple[int, int]:
    """(max_node_len, nodes_per_page) the way DiskANN lays records out."""
    node_len = num_dims * elem + 4 * (max_m0 + 1)
    if node_len > PAGE_SIZE:
        raise ValueError("record larger than a 4 KB page")
    return node_len, PAGE_SIZE // node_len


def _rows(x, a: int, b: int) -> np.ndarray:
    """Rows [a, b) of a numpy array or a (possibly CUDA) torch tensor, as numpy."""
    if hasattr(x, "detach"):
        return x[a:b].detach().cpu().numpy()
    return np.asarray(x[a:b])


def write_disk_index(path: str, vectors, adj, deg, medoid: int, max_m0: int | None = None,
                     chunk_pages: int = 1 << 16) -> DiskLayout:
    """Write records ``[T x D vector][u32 deg][u32 nbr x max_m0]`` into 4 KB pages.

    ``adj`` is ``[N, >=max(deg)]`` int; entries past ``deg`` are ignored (zero-filled
    on disk). The header is DiskANN's metadata ``bin<u64>`` (9 values).
    ``vectors``, ``adj`` and ``deg`` may be numpy arrays or torch tensors (also on
    a GPU); the file is written ``chunk_pages`` pages at a time, so host memory
    stays bounded at any N.
    """
    n, d = vectors.shape
    elem = np.dtype(str(vectors.dtype).replace("torch.", "")).itemsize
    if max_m0 is None:
        max_m0 = int(adj.shape[1])
    node_len, npp = record_geometry(d, elem, max_m0)
    num_pages = (n + npp - 1) // npp
    file_size = (num_pages + 1) * PAGE_SIZE

    meta = np.array([n, d, medoid, node_len, npp, 0, 0, 0, file_size], dtype=np.uint64)
    header = np.zeros(PAGE_SIZE, dtype=np.uint8)
    hb = struct.pack("<II", len(meta), 1) + meta.tobytes()
    header[: len(hb)] = np.frombuffer(hb, dtype=np.uint8)
    w = min(max_m0, adj.shape[1])
    with open(path, "wb") as f:
        f.write(header.tobytes())
        for p0 in range(0, num_pages, chunk_pages):
            p1 = min(num_pages, p0 + chunk_pages)
            r0, r1 = p0 * npp, min(n, p1 * npp)
            m = r1 - r0
            rec = np.zeros(((p1 - p0) * npp, node_len), dtype=np.uint8)
            rec[:m, : d * elem] = np.ascontiguousarray(_rows(vectors, r0, r1)).view(np.uint8).reshape(m, d * elem)
            dg = _rows(deg, r0, r1).astype(np.uint32)
            a = _rows(adj, r0, r1)[:, :w]
            nb = np.zeros((m, max_m0), dtype=np.uint32)
            nb[:, :w] = np.where(np.arange(w)[None, :] < dg[:, None], a, 0).astype(np.uint32)
            rec[:m, d * elem: d * elem + 4] = dg.reshape(m, 1).view(np.uint8)
            rec[:m, d * elem + 4:] = nb.view(np.uint8)
            pages = np.zeros((p1 - p0, PAGE_SIZE), dtype=np.uint8)
            pages[:, : npp * node_len] = rec.reshape(p1 - p0, npp * node_len)
            f.write(pages.tobytes())
    return DiskLayout(n, d, medoid, node_len, npp, d * elem, max_m0, num_pages)


def read_disk_header(path: str, elem: int) -> DiskLayout:
    """Mirror of ``Layout::parse_diskann_metadata`` (``src/layout.cpp:11-69``)."""
    with open(path, "rb") as f:
        nr, nc = struct.unpack("<II", f.read(8))
        vals = struct.unpack("<8Q", f.read(64))
    n, d, medoid, node_len, npp = vals[:5]
    data_size = d * elem
    max_m0 = (node_len - data_size) // 4 - 1
    return DiskLayout(int(n), int(d), int(medoid), int(node_len), int(npp), int(data_size),
                      int(max_m0), int((n + npp - 1) // npp))


def read_disk_index(path: str, dtype: int):
    """Return (layout, vectors [N,D], deg [N], nbrs [N,max_m0]) from a disk index."""
    t = np_dtype(dtype)
    lay = read_disk_header(path, np.dtype(t).itemsize)
    raw = np.fromfile(path, dtype=np.uint8, offset=PAGE_SIZE)
    raw = raw[: lay.num_pages * PAGE_SIZE].reshape(lay.num_pages, PAGE_SIZE)
    rec = raw[:, : lay.nodes_per_page * lay.max_node_len].reshape(-1, lay.max_node_len)[: lay.num_data]
    vec = rec[:, : lay.data_size].copy().view(t).reshape(lay.num_data, lay.num_dims)
    deg = rec[:, lay.data_size: lay.data_size + 4].copy().view(np.uint32).reshape(-1)
    nbrs = rec[:, lay.data_size + 4:].copy().view(np.uint32).reshape(lay.num_data, lay.max_m0)
    return lay, vec, deg, nbrs


# ------------------------------------------------------------------------- PQ


def chunk_offsets_for(dim: int, m: int) -> np.ndarray:
    """Contiguous chunks; the first ``dim % m`` chunks take one extra dimension."""
    if not 0 < m <= dim:
        raise ValueError("need 0 < M <= dim")
    lo, extra = divmod(dim, m)
    sizes = np.array([lo + 1] * extra + [lo] * (m - extra), dtype=np.uint32)
    return np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)


def write_pq(prefix: str, pivots: np.ndarray, centroid: np.ndarray,
             chunk_offsets: np.ndarray, codes: np.ndarray, legacy: bool = False) -> None:
    """``<prefix>_pivots.bin`` (offsets table + 3 bins) and ``<prefix>_compressed.bin``.

    New-DiskANN layout (``nr == 4``) puts the chunk offsets in the third slot; the
    legacy/PipeANN layout (``nr == 5``) has an extra slot before it
    (``src/pq_search.cu:78-117``).
    """
    piv = prefix + "_pivots.bin"
    assert pivots.shape[0] == NUM_PIVOTS
    offs = [PAGE_SIZE]
    with open(piv, "wb") as f:
        f.write(b"\0" * PAGE_SIZE)
    offs.append(offs[-1] + write_bin(piv, pivots.astype(np.float32), offs[-1]))
    offs.append(offs[-1] + write_bin(piv, centroid.astype(np.float32).reshape(-1, 1), offs[-1]))
    if legacy:
        # the retired "rearrangement" slot: an identity permutation
        perm = np.arange(pivots.shape[1], dtype=np.uint32).reshape(-1, 1)
        offs.append(offs[-1] + write_bin(piv, perm, offs[-1]))
    offs.append(offs[-1] + write_bin(piv, chunk_offsets.astype(np.uint32).reshape(-1, 1), offs[-1]))
    write_bin(piv, np.array(offs, dtype=np.uint64).reshape(-1, 1), 0)
    write_bin(prefix + "_compressed.bin", np.ascontiguousarray(codes.astype(np.uint8)))


def read_pq(prefix: str):
    """Return (pivots [256,D], centroid [D], chunk_offsets [M+1], codes [N,M])."""
    piv = prefix + "_pivots.bin"
    offs = read_bin(piv, np.uint64, 0).reshape(-1)
    nr = offs.size
    if nr not in (4, 5):
        raise ValueError(f"{piv}: offsets table has {nr} rows")
    pivots = read_bin(piv, np.float32, int(offs[0]))
    centroid = read_bin(piv, np.float32, int(offs[1])).reshape(-1)
    chunk = read_bin(piv, np.uint32, int(offs[3] if nr == 5 else offs[2])).reshape(-1)
    codes = read_bin(prefix + "_compressed.bin", np.uint8, 0)
    return pivots, centroid, chunk, codes


# ------------------------------------------------------------------ nav graph


def write_nav(directory: str, sample_vectors: np.ndarray, sample_ids: np.ndarray,
              adj: np.ndarray, deg: np.ndarray, start: int, max_degree: int | None = None) -> None:
    """Write the pivot-graph directory the reference loads (``src/nav_graph.cu:41-100``).

    ``nav_index`` is DiskANN's in-memory graph: ``u64 file_size, u32 max_degree,
    u32 start, u64 num_frozen`` then per node ``u32 d, u32 nbr[d]``.
    ``nav_index.data`` is a ``bin`` of the sampled vectors; ``map.txt`` holds the
    global id of each sample, one per line. ``max_degree`` is the row width the
    header announces (defaults to the largest degree present).
    """
    os.makedirs(directory, exist_ok=True)
    s = sample_vectors.shape[0]
    deg = np.asarray(deg, dtype=np.uint32)
    max_deg = int(deg.max()) if s else 0
    if max_degree is not None:
        if max_degree < max_deg:
            raise ValueError("max_degree below the largest node degree")
        max_deg = max_degree
    # per node: u32 degree, then its first `degree` neighbour ids
    adj = np.asarray(adj)
    w = adj.shape[1] if adj.ndim == 2 else 0
    if s and int(deg.max()) > w:
        raise ValueError("a degree exceeds the adjacency width")
    keep = np.arange(w)[None, :] < deg[:, None] if s else np.zeros((0, 0), bool)
    body = np.zeros(s + int(deg.sum()), dtype=np.uint32)
    starts = np.arange(s, dtype=np.int64) + np.concatenate([[0], np.cumsum(deg, dtype=np.int64)[:-1]]) if s else \
        np.zeros(0, np.int64)
    body[starts] = deg
    if s:
        slot = starts[:, None] + 1 + np.arange(w)[None, :]
        body[slot[keep]] = adj[keep].astype(np.uint32)
    size = 24 + 4 * body.size
    with open(os.path.join(directory, "nav_index"), "wb") as f:
        f.write(struct.pack("<QIIQ", size, max_deg, int(start), 0))
        f.write(body.tobytes())
    write_bin(os.path.join(directory, "nav_index.data"), np.ascontiguousarray(sample_vectors))
    with open(os.path.join(directory, "map.txt"), "w") as f:
        f.write("".join(f"{int(x)}\n" for x in sample_ids))


def read_nav(directory: str, dtype: int):
    """Return (vectors [S,D], adj [S,max_m] padded with -1, start, map [S])."""
    t = np_dtype(dtype)
    vec = read_bin(os.path.join(directory, "nav_index.data"), t, 0)
    ids = np.loadtxt(os.path.join(directory, "map.txt"), dtype=np.int64, ndmin=1).astype(np.int32)
    raw = np.fromfile(os.path.join(directory, "nav_index"), dtype=np.uint8)
    _, max_m, start, _ = struct.unpack("<QIIQ", raw[:24].tobytes())
    words = raw[24:].view(np.uint32)
    s = vec.shape[0]
    adj = np.full((s, max_m), -1, dtype=np.int32)
    p = 0
    for i in range(s):
        k = int(words[p])
        adj[i, :k] = words[p + 1: p + 1 + k].view(np.int32)
        p += 1 + k
    return vec, adj, int(start), ids


def index_paths(root: str) -> dict:
    """Canonical file names under one index directory (``src/ssd_search.cu:55-79``)."""
    return {
        "index_file": os.path.join(root, "index_disk.index"),
        "pq_file_prefix": os.path.join(root, "index_pq"),
        "nav_graph_prefix": os.path.join(root, "nav"),
        "query_file": os.path.join(root, "query"),
        "gt_file": os.path.join(root, "gt.ivecs"),
    }
