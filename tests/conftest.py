"""Shared fixtures: small seeded indexes built once per session.

GPU tests are marked ``gpu`` and skipped when no CUDA device is visible.
"""
import os
import sys
import tempfile

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

from gustann_b200 import formats  # noqa: E402
from gustann_b200.index import datagen, pipeline  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def has_gpu() -> bool:
    return torch.cuda.is_available()


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


# name -> (mixture spec, R, M, nav samples, nav?)
INDEXES = {
    "u8": (datagen.MixtureSpec("sift", 12000, 128, 60, 20.0), 32, 32, 1500, True),
    # configurations 0/2/3's shape: uint8, 128 dims, R = 64, M = 32 (4 dims a chunk)
    "u8_r64": (datagen.MixtureSpec("sift", 16000, 128, 80, 20.0), 64, 32, 2000, True),
    "f32": (datagen.MixtureSpec("deep", 12000, 96, 60, 0.1, center_scale=0.15), 64, 32, 1500, True),
    "f32_odd": (datagen.MixtureSpec("deep", 4000, 40, 20, 0.1, center_scale=0.15), 96, 12, 500, True),
    "u8_nonav": (datagen.MixtureSpec("sift", 6000, 64, 30, 20.0), 48, 16, 0, False),
    # configuration-4 shape: 768 dims, 96 PQ chunks of 8 dims (per-query tables)
    "f32_wide": (datagen.MixtureSpec("deep", 3000, 768, 20, 0.1, center_scale=0.15), 64, 96, 400, True),
}


# inner-product indexes (searched with GANN_METRIC_IP; the graph is built on
# L2 over unit vectors, where both orders agree): configuration 4's text-like
# mixture with Zipf(1.1) queries, at 96 dims (pivot-mode ADC) and at
# configuration 4's own shape, 768 dims in 96 chunks of 8 (per-query tables)
IP_INDEXES = {
    "ip96": (datagen.MixtureSpec("text", 8000, 96, 40, 0.1, center_scale=0.15, zipf=1.1, query_noise=0.05),
             64, 32, 1000, True),
    "ip768": (datagen.MixtureSpec("text", 3000, 768, 20, 0.1 * (96 / 768) ** 0.5, center_scale=768 ** -0.5,
                                  zipf=1.1, query_noise=0.05), 64, 96, 400, True),
}


@pytest.fixture(scope="session")
def index_root():
    d = os.environ.get("GANN_TEST_INDEX_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return tempfile.mkdtemp(prefix="gann_test_idx_")


_built = {}


def get_index(root: str, name: str) -> dict:
    """Build (once) and return paths + queries of a named test index."""
    if name in _built:
        return _built[name]
    spec, R, M, nav_s, nav = INDEXES[name] if name in INDEXES else IP_INDEXES[name]
    d = os.path.join(root, name)
    paths = formats.index_paths(d)
    dev = "cuda" if has_gpu() else "cpu"
    if not os.path.exists(os.path.join(d, "meta.json")):
        X = datagen.base_vectors(spec, device=dev)
        paths = pipeline.build_index(d, X, spec.dtype, R=R, M=M, nav_samples=max(nav_s, 1), nav=nav)
    elif not nav:
        paths["nav_graph_prefix"] = ""
    q = datagen.as_float_queries(datagen.query_vectors(spec, 400, device="cpu"))
    info = {"paths": paths, "queries": q, "dtype": spec.dtype, "dim": spec.dim, "R": R, "M": M, "spec": spec}
    _built[name] = info
    return info


@pytest.fixture(scope="session", params=list(INDEXES))
def any_index(request, index_root):
    return get_index(index_root, request.param)
