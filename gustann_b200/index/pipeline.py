"""Build a complete search index (disk index + PQ + pivot graph) from vectors.

The produced directory is what the reference's loaders read (file names of
``scripts/build_diskann_index.sh`` / ``scripts/gen_pivot_graph.sh``):

  <root>/index_disk.index            DiskANN disk index (records in 4 KB pages)
  <root>/index_pq_pivots.bin         PQ pivots, centroid, chunk offsets
  <root>/index_pq_compressed.bin     PQ codes
  <root>/nav/{nav_index, nav_index.data, map.txt}   pivot graph

Steps mirror the reference's index preparation: graph build (R, alpha), PQ
training with M chunks, then a pivot sample of ``min(N, nav_samples)`` points
chosen like ``bin/gen_small_file.cpp`` (std::shuffle with mt19937(114514), ids
sorted) and a degree-32 graph over the sample (``scripts/gen_pivot_graph.sh:12-13``).
"""
from __future__ import annotations

import json
import os
import time

import numpy as np
import torch

from .. import formats
from .graph import build_graph, medoid
from .pq import encode_pq, train_pq

NAV_DEGREE = 32
PIVOT_SEED = 114514


def _to_numpy(x: torch.Tensor, dtype: int) -> np.ndarray:
    return x.cpu().numpy().astype(formats.np_dtype(dtype), copy=False)


def sample_pivots(n: int, s: int) -> np.ndarray:
    """Pivot-graph sample ids, drawn by the native library's std::shuffle."""
    from ..api import pivot_sample
    return pivot_sample(n, s, PIVOT_SEED)


def build_index(root: str, X: torch.Tensor, dtype: int, R: int = 64, alpha: float = 1.2, M: int = 32,
                nav_samples: int = 1_000_000, nav: bool = True, seed: int = 0, verbose: bool = False,
                pq_legacy: bool = False, long_range: int = 4, L_build: int = 100, nav_L: int = 50,
                builder: str = "auto", passes: int = 2) -> dict:
    """Build every index file under ``root`` for base vectors ``X`` [N, D].

    ``builder``: "vamana" (GPU; greedy-search candidates, the construction the
    reference's indexes come from), "knn" (kNN + RobustPrune; CPU or GPU), or
    "auto" (vamana when ``X`` is on a GPU). Returns the path dict of
    :func:`gustann_b200.formats.index_paths` plus timings.
    """
    os.makedirs(root, exist_ok=True)
    paths = formats.index_paths(root)
    t = {}
    n = X.shape[0]
    use_vamana = builder == "vamana" or (builder == "auto" and X.is_cuda)

    t0 = time.time()
    pivots, centroid, offs = train_pq(X, M, seed=seed)
    codes = encode_pq(X, pivots, centroid, offs)
    formats.write_pq(paths["pq_file_prefix"], pivots, centroid, offs, codes, legacy=pq_legacy)
    t["pq_s"] = time.time() - t0

    def graph(Xg, codes_g, R_g, L_g, seed_g):
        if use_vamana:
            from .vamana import vamana_graph
            a, d, m = vamana_graph(Xg, codes_g, pivots, centroid, offs, R=R_g, L=L_g, alpha=alpha,
                                   passes=passes, seed=seed_g, verbose=verbose)
            return a, d, m
        a, d = build_graph(Xg, R_g, alpha=alpha, seed=seed_g, long_range=long_range)
        return a, d, medoid(Xg)

    t0 = time.time()
    adj, deg, med = graph(X, codes, R, L_build, seed)
    t["graph_s"] = time.time() - t0
    if verbose:
        print(f"[index] graph n={n} R={R}: {t['graph_s']:.1f}s, mean degree {float(deg.float().mean()):.1f}",
              flush=True)

    t0 = time.time()
    formats.write_disk_index(paths["index_file"], X, adj, deg, med, max_m0=R)
    t["write_s"] = time.time() - t0

    if nav:
        t0 = time.time()
        s = min(n, nav_samples)
        ids = sample_pivots(n, s)
        Xs = X[torch.from_numpy(ids.astype(np.int64)).to(X.device)]
        nadj, ndeg, start = graph(Xs, codes[ids], NAV_DEGREE, nav_L, seed + 1)
        formats.write_nav(paths["nav_graph_prefix"], _to_numpy(Xs, dtype), ids, nadj.cpu().numpy(),
                          ndeg.cpu().numpy(), start, max_degree=NAV_DEGREE)
        t["nav_s"] = time.time() - t0
    else:
        paths["nav_graph_prefix"] = ""
    meta = {"n": int(n), "dim": int(X.shape[1]), "dtype": int(dtype), "R": R, "alpha": alpha, "M": M,
            "medoid": int(med), "builder": "vamana" if use_vamana else "knn", "timings": t}
    with open(os.path.join(root, "meta.json"), "w") as f:
        json.dump(meta, f)
    paths["meta"] = meta
    return paths
