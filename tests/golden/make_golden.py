"""Generate the golden fixtures that pin the CPU oracle to the reference.

Two steps (the committed fixtures are the output of both):

1. ``python tests/golden/make_golden.py --index``  (any machine, CPU)
   writes two tiny seeded indexes (uint8 and float32) plus their queries under
   ``tests/golden/<name>/``.
2. ``python tests/golden/make_golden.py --ref OUT``  (a machine with a GPU and
   ``oracle/_ref/libgustann_ref.so`` built from the reference's own sources)
   runs the reference's kernels on those files and writes ``OUT/<name>/ref.npz``
   (ADC tables, pivot-graph entries, search results for several ``ef``); copy
   them next to the index files.

The reference ships no golden vectors or tests of its own, so these outputs of
its compiled kernels are the known answers the oracle is checked against.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

GOLDEN = {
    # name: (kind, n, dim, centers, sigma, center_scale, R, M, nav samples)
    "g_u8": ("sift", 2000, 32, 12, 20.0, 1.0, 24, 8, 300),
    "g_f32": ("deep", 2000, 24, 12, 0.1, 0.2, 24, 8, 300),
}
EFS = (10, 20, 40)
TOPK = 10
NQ = 64


def paths(name: str) -> dict:
    from gustann_b200 import formats
    return formats.index_paths(os.path.join(HERE, name))


def make_index() -> None:
    import torch
    from gustann_b200.index import datagen, pipeline
    torch.set_num_threads(1)
    for name, (kind, n, dim, c, sig, cs, R, M, S) in GOLDEN.items():
        spec = datagen.MixtureSpec(kind, n, dim, c, sig, center_scale=cs)
        X = datagen.base_vectors(spec, "cpu")
        d = os.path.join(HERE, name)
        pipeline.build_index(d, X, spec.dtype, R=R, M=M, nav_samples=S, long_range=2)
        q = datagen.as_float_queries(datagen.query_vectors(spec, NQ, "cpu"))
        np.save(os.path.join(d, "queries.npy"), q)
        print("wrote", d)


def make_ref(out: str) -> None:
    from oracle import RefGPU
    os.makedirs(out, exist_ok=True)
    for name, (kind, n, dim, c, sig, cs, R, M, S) in GOLDEN.items():
        p = paths(name)
        q = np.load(os.path.join(HERE, name, "queries.npy"))
        dtype = 0 if kind == "sift" else 1
        # the reference only gets inputs inside its defined behaviour
        from oracle import Oracle
        o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], dtype)
        for ef in EFS:
            assert not o.search(q, TOPK, ef)[4].any(), "golden queries must be flag-free"
        r = RefGPU(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], dtype, dim)
        res = {"lut": r.lut(q[:8], M)}
        res["nav_sample"], res["nav_entry"] = r.nav(q)
        for ef in EFS:
            nns, dist, found, _ = r.search(q, TOPK, ef)
            res[f"nns_{ef}"], res[f"dist_{ef}"], res[f"found_{ef}"] = nns, dist, found
        r.close()
        os.makedirs(os.path.join(out, name), exist_ok=True)
        np.savez_compressed(os.path.join(out, name, "ref.npz"), **res)
        print("wrote", os.path.join(out, name, "ref.npz"))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--index", action="store_true")
    ap.add_argument("--ref", metavar="OUT")
    a = ap.parse_args()
    if a.index:
        make_index()
    if a.ref:
        make_ref(a.ref)
