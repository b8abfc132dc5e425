"""Build one benchmark configuration's index, queries and ground truth.

  python -m gustann_b200.index.make --config c2 --root DIR [--points N] [--nq Q]

Writes under ``DIR`` the index files the reference's loaders read (see
:mod:`gustann_b200.index.pipeline`), the query set in the reference driver's
format (``query.bvecs`` for uint8 data, ``query.fvecs`` for float32;
``bin/utils.hpp:23-88``), the exact top-``k`` of every query (``gt.ivecs``,
brute force on the GPU with ``gann_exact_knn``), ``meta.json`` with the build
timings, and last a ``DONE`` marker. A directory holding ``DONE`` is complete;
callers wait for it.

It runs as its own process so that a caller which must not load this
library (the benchmark's reference arm) can still have the index built.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import time

import numpy as np
import torch

from .. import formats
from . import datagen, pipeline

# index parameters per configuration (R, PQ chunks, metric, top-k of the GT)
PARAMS = {
    "c0": dict(R=64, M=32, metric=0, k=10),
    "c1": dict(R=64, M=32, metric=0, k=10),
    "c2": dict(R=64, M=32, metric=0, k=10),
    "c3": dict(R=64, M=32, metric=0, k=10),
    "c4": dict(R=64, M=96, metric=1, k=100),
}


def query_file(root: str, dtype: int) -> str:
    return os.path.join(root, "query.bvecs" if dtype == formats.UINT8 else "query.fvecs")


def read_queries(root: str, dtype: int) -> np.ndarray:
    """The query set as float32 rows (uint8 queries widened, as the
    reference's driver does, bin/search_disk.cpp:160-165)."""
    q = formats.read_vecs(query_file(root, dtype), formats.np_dtype(dtype))
    return q.astype(np.float32)


def ground_truth(X: torch.Tensor, Q: torch.Tensor, k: int, metric: int, block: int = 25_000) -> np.ndarray:
    from ..api import exact_knn
    out = []
    for s in range(0, Q.shape[0], block):
        ids, _ = exact_knn(X, Q[s: s + block].contiguous(), k, metric)
        out.append(ids.cpu().numpy())
    return np.concatenate(out) if out else np.zeros((0, k), np.int32)


def make(config: str, root: str, n: int = 0, nq: int = 10_000, passes: int = 2, nav_samples: int = 1_000_000,
         verbose: bool = True, order: str = "input") -> dict:
    spec = datagen.CONFIGS[config]
    spec = dataclasses.replace(spec, n=n or spec.n)
    p = PARAMS[config]
    os.makedirs(root, exist_ok=True)
    t = {}
    t0 = time.time()
    X = datagen.base_vectors(spec, device="cuda")
    torch.cuda.synchronize()
    t["datagen_s"] = time.time() - t0
    if order == "partition":
        # rows grouped by coarse partition (reorder.py); ids.bin maps each
        # index row to its generated row, and the ground truth and search
        # results both use index rows
        from .reorder import partition_order
        t0 = time.time()
        perm = partition_order(X)
        X = X[perm]
        perm.to(torch.int32).cpu().numpy().tofile(os.path.join(root, "ids.bin"))
        del perm
        torch.cuda.synchronize()
        t["order_s"] = time.time() - t0
    paths = pipeline.build_index(root, X, spec.dtype, R=p["R"], alpha=1.2, M=p["M"], nav_samples=nav_samples,
                                 passes=passes, verbose=verbose)
    t.update(paths["meta"]["timings"])
    t0 = time.time()
    Q = datagen.query_vectors(spec, nq, device="cuda", offset=0)
    formats.write_vecs(query_file(root, spec.dtype), Q.cpu().numpy())
    gt = ground_truth(X, Q, p["k"], p["metric"])
    formats.write_vecs(os.path.join(root, "gt.ivecs"), gt.astype(np.int32))
    torch.cuda.synchronize()
    t["gt_s"] = time.time() - t0
    meta = dict(paths["meta"], config=config, nq=nq, gt_k=p["k"], metric=p["metric"], passes=passes, order=order,
                spec=dataclasses.asdict(spec), timings=t)
    with open(os.path.join(root, "meta.json"), "w") as f:
        json.dump(meta, f)
    with open(os.path.join(root, "DONE"), "w") as f:
        f.write(json.dumps(t) + "\n")
    if verbose:
        print(f"[make] {config} n={spec.n} done: " + ", ".join(f"{k} {v:.1f}" for k, v in t.items()), flush=True)
    return meta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2", choices=list(datagen.CONFIGS))
    ap.add_argument("--root", required=True)
    ap.add_argument("--points", type=int, default=0)
    ap.add_argument("--nq", type=int, default=10_000)
    ap.add_argument("--passes", type=int, default=2)
    ap.add_argument("--nav-samples", type=int, default=1_000_000)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--order", default="input", choices=["input", "partition"],
                    help="record order: as generated, or grouped by coarse partition (reorder.py)")
    a = ap.parse_args()
    torch.cuda.set_device(a.device)
    make(a.config, a.root, a.points, a.nq, a.passes, a.nav_samples, order=a.order)


if __name__ == "__main__":
    main()
