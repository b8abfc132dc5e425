"""The CPU oracle: pinned to the reference's own kernel outputs (golden
fixtures produced on a B200 by tests/golden/make_golden.py) and checked for
the properties the reference's algorithm guarantees."""
import os

import numpy as np
import pytest

from conftest import ROOT, get_index
from gustann_b200 import formats
from gustann_b200.index.graph import knn_exact
from oracle import F_NAVRACE, Oracle

GOLD = os.path.join(ROOT, "tests", "golden")
NAMES = {"g_u8": formats.UINT8, "g_f32": formats.FLOAT}


def _golden(name):
    npz = os.path.join(GOLD, name, "ref.npz")
    if not os.path.exists(npz):
        pytest.skip("reference outputs not generated yet")
    p = formats.index_paths(os.path.join(GOLD, name))
    q = np.load(os.path.join(GOLD, name, "queries.npy"))
    return p, q, np.load(npz)


@pytest.mark.parametrize("name", list(NAMES))
def test_oracle_lut_equals_reference(name):
    p, q, ref = _golden(name)
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], NAMES[name], fma_mode=1)
    np.testing.assert_array_equal(o.lut(q[: len(ref["lut"])]), ref["lut"])


@pytest.mark.parametrize("name", list(NAMES))
def test_oracle_nav_equals_reference(name):
    p, q, ref = _golden(name)
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], NAMES[name])
    s, e, f = o.nav(q)
    assert not (f & F_NAVRACE).any()
    np.testing.assert_array_equal(s, ref["nav_sample"])
    np.testing.assert_array_equal(e, ref["nav_entry"])


@pytest.mark.parametrize("name", list(NAMES))
@pytest.mark.parametrize("ef", [10, 20, 40])
def test_oracle_search_equals_reference(name, ef):
    p, q, ref = _golden(name)
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], NAMES[name])
    nns, dist, found, hops, flags = o.search(q, 10, ef)
    assert not flags.any()
    np.testing.assert_array_equal(found, ref[f"found_{ef}"])
    np.testing.assert_array_equal(nns, ref[f"nns_{ef}"])
    np.testing.assert_array_equal(dist, ref[f"dist_{ef}"])


def test_fma_contraction_matters_and_is_pinned():
    """The reference's `acc += d*d` is contracted to fma by nvcc; the separate
    multiply-add variant gives different tables on the f32 fixture."""
    p, q, ref = _golden("g_f32")
    o0 = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.FLOAT, fma_mode=0)
    assert not np.array_equal(o0.lut(q[:8]), ref["lut"])


def test_lut_close_to_float64():
    info_dir = os.path.join(GOLD, "g_f32")
    p = formats.index_paths(info_dir)
    q = np.load(os.path.join(info_dir, "queries.npy"))[:4]
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.FLOAT)
    piv, cen, offs, _ = formats.read_pq(p["pq_file_prefix"])
    lut = o.lut(q)
    r = q.astype(np.float64) - cen
    for c in range(len(offs) - 1):
        a, b = offs[c], offs[c + 1]
        exact = ((r[:, None, a:b] - piv[None, :, a:b].astype(np.float64)) ** 2).sum(-1)
        np.testing.assert_allclose(lut[:, c, :], exact, rtol=1e-5, atol=1e-6)


def test_results_are_sorted_exact_distances():
    p = formats.index_paths(os.path.join(GOLD, "g_u8"))
    q = np.load(os.path.join(GOLD, "g_u8", "queries.npy"))
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.UINT8)
    nns, dist, found, hops, flags = o.search(q, 10, 40)
    _, vec, _, _ = formats.read_disk_index(p["index_file"], formats.UINT8)
    assert np.all(found == 10) and np.all(hops >= 10)
    assert np.all(np.diff(dist, axis=1) >= 0)
    exact = ((vec[nns].astype(np.float64) - q[:, None, :]) ** 2).sum(-1)
    np.testing.assert_allclose(dist, exact, rtol=1e-6)


def test_recall_improves_with_ef(index_root):
    info = get_index(index_root, "u8")
    p = info["paths"]
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"])
    q = info["queries"][:200]
    _, vec, _, _ = formats.read_disk_index(p["index_file"], info["dtype"])
    import torch
    gt = knn_exact(torch.from_numpy(vec.astype(np.float32)), torch.from_numpy(q), 10)[0].numpy()
    recs = []
    for ef in (10, 40, 160):
        nns = o.search(q, 10, ef)[0]
        recs.append(np.mean([len(set(a) & set(b)) for a, b in zip(nns, gt)]) / 10)
    assert recs[0] <= recs[1] <= recs[2] and recs[2] > 0.9, recs


def test_ip_oracle_definitions():
    """Inner product (no reference counterpart): table entries are
    -(q . pivot) per chunk, exact distances -<q, x>, results ascending."""
    p = formats.index_paths(os.path.join(GOLD, "g_f32"))
    q = np.load(os.path.join(GOLD, "g_f32", "queries.npy"))[:16]
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.FLOAT, metric=1)
    piv, cen, offs, _ = formats.read_pq(p["pq_file_prefix"])
    lut = o.lut(q[:4])
    for c in range(len(offs) - 1):
        a, b = offs[c], offs[c + 1]
        exact = -(q[:4, None, a:b].astype(np.float64) * piv[None, :, a:b].astype(np.float64)).sum(-1)
        np.testing.assert_allclose(lut[:, c, :], exact, rtol=1e-5, atol=1e-6)
    nns, dist, found, hops, flags = o.search(q, 10, 40)
    _, vec, _, _ = formats.read_disk_index(p["index_file"], formats.FLOAT)
    assert np.all(np.diff(dist, axis=1) >= 0)
    exact = -np.einsum("qd,qkd->qk", q.astype(np.float64), vec[nns].astype(np.float64))
    np.testing.assert_allclose(dist, exact, rtol=1e-5, atol=1e-6)
    # the L2 search of the same oracle differs (another metric, another order)
    o2 = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.FLOAT)
    assert not np.array_equal(o2.search(q, 10, 40)[1], dist)
