"""Host-driven search, one hop per call (the reference's SSD-hybrid mode):
node records stay in the index file, the caller reads the 4 KB page of every
query's next node between hops (gann_read_pages), the GPU does the ADC, merge
and re-rank. Results must equal the oracle's with the hybrid mode's entry: the
pivot-graph search on q'' = (q - c) + c (src/hyd_task_runner.cu:55-66).

The page loader is host code and is tested without a GPU.
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, get_index
from gustann_b200 import api, formats
from gustann_b200.api import GustANN, GustANNConfig, GustANNError, GustANNStats
from oracle import F_NAVRACE, Oracle

GOLD = os.path.join(ROOT, "tests", "golden", "g_u8")


def _lay(path, dtype):
    lay, _, _, _ = formats.read_disk_index(path, dtype)
    return lay


# ------------------------------------------------------------------ CPU
def test_read_pages_matches_the_file():
    p = formats.index_paths(GOLD)
    f = p["index_file"]
    lay = _lay(f, formats.UINT8)
    npp = lay.nodes_per_page
    ids = np.array([0, 5, -1, lay.num_data - 1, 17, 17], np.int32)
    pages = np.full((len(ids), 4096), 7, np.uint8)
    assert api.lib.gann_read_pages(f.encode(), api._ptr(ids), len(ids), npp, api._ptr(pages), 3) == api.GANN_OK
    raw = open(f, "rb").read()
    for i, u in enumerate(ids):
        if u < 0:
            assert np.all(pages[i] == 7)          # untouched
        else:
            off = 4096 * (1 + u // npp)
            assert bytes(pages[i]) == raw[off: off + 4096]


def test_read_pages_errors(tmp_path):
    p = formats.index_paths(GOLD)
    f = p["index_file"]
    npp = _lay(f, formats.UINT8).nodes_per_page
    pages = np.zeros((1, 4096), np.uint8)
    far = np.array([10 ** 8], np.int32)
    assert api.lib.gann_read_pages(f.encode(), api._ptr(far), 1, npp, api._ptr(pages), 1) == api.GANN_EIO
    missing = str(tmp_path / "nope").encode()
    ok = np.array([0], np.int32)
    assert api.lib.gann_read_pages(missing, api._ptr(ok), 1, npp, api._ptr(pages), 1) == api.GANN_EIO
    assert api.lib.gann_read_pages(f.encode(), None, 1, npp, None, 1) == api.GANN_EINVAL


def test_hop_calls_reject_bad_arguments():
    assert api.lib.gann_hop_begin(None, None, 0, 10, 10, None) == api.GANN_EINVAL
    assert api.lib.gann_hop_requests(None, None, None) == api.GANN_EINVAL
    assert api.lib.gann_hop_step(None, None) == api.GANN_EINVAL
    assert api.lib.gann_hop_finish(None, None, None, None) == api.GANN_EINVAL
    assert api.lib.gann_hop_free(None) == api.GANN_OK


# ------------------------------------------------------------------ GPU
def _hybrid_oracle(info, q, topk, ef):
    """Oracle search entered where the hybrid mode enters: nav on q''."""
    p = info["paths"]
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"])
    try:
        entries = None
        navflags = np.zeros(len(q), np.int32)
        if p["nav_graph_prefix"]:
            _, cen, _, _ = formats.read_pq(p["pq_file_prefix"])
            cen = cen.astype(np.float32).reshape(-1)
            qpp = ((q - cen).astype(np.float32) + cen).astype(np.float32)
            _, entries, navflags = o.nav(qpp)
        res = o.search(q, topk, ef, entries=entries)
    finally:
        o.close()
    return res, navflags


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["u8", "f32", "f32_odd", "u8_nonav"])
@pytest.mark.parametrize("ef", [10, 64, 200])
def test_hop_search_equals_oracle(index_root, name, ef):
    info = get_index(index_root, name)
    p = info["paths"]
    g = GustANN(info["dtype"])
    g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), True)
    q = info["queries"][:200]
    try:
        nns, dist, found, rounds = g.hop_search(q, 10, ef, index_file=p["index_file"], threads=4)
    finally:
        g.close()
    (onns, odist, ofound, ohops, oflags), navflags = _hybrid_oracle(info, q, 10, ef)
    ok = ((oflags | navflags) & F_NAVRACE) == 0
    np.testing.assert_array_equal(nns[ok], onns[ok])
    np.testing.assert_array_equal(dist[ok], odist[ok])
    np.testing.assert_array_equal(found[ok], ofound[ok])
    assert rounds >= int(ohops[ok].max())


@pytest.mark.gpu
def test_init_hybrid_keeps_records_on_storage(index_root):
    info = get_index(index_root, "f32")
    p = info["paths"]
    cfg = GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"])
    mem = GustANN(info["dtype"])
    mem.init_pure_mem(cfg, True)
    hyb = GustANN(info["dtype"])

    class HC:                      # HybridExecutorConfig fields that apply
        mini_batch = 64
        thread_cnt = 4

    hyb.init_hybrid(cfg, HC())
    q = info["queries"][:150]
    try:
        assert hyb.info()["device_bytes"] < mem.info()["device_bytes"]
        st = GustANNStats()
        a = hyb.query(q, 10, 64, st)
        b = hyb.hop_search(q, 10, 64)[:3]
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)
        assert st.hops > 0
        # the in-HBM search refuses a handle without records
        nns = np.zeros((len(q), 10), np.int32)
        dst = np.zeros((len(q), 10), np.float32)
        fnd = np.zeros(len(q), np.int32)
        rc = api.lib.gann_search(hyb._h, api._ptr(np.ascontiguousarray(q)), len(q), 10, 64, api._ptr(nns),
                                 api._ptr(dst), api._ptr(fnd), None)
        assert rc == api.GANN_ESTATE
    finally:
        mem.close()
        hyb.close()


@pytest.mark.gpu
def test_cli_hybrid_mode(index_root, tmp_path):
    """search_mem --hybrid (the reference driver's HYBRID_CALC build) runs as
    the in-HBM mode does; its recall against the hybrid search's own results
    is 1."""
    info = get_index(index_root, "u8")
    p = info["paths"]
    q = info["queries"][:100]
    qf, gf = tmp_path / "q.bvecs", tmp_path / "gt.ivecs"
    formats.write_vecs(str(qf), q.astype(np.uint8))
    g = GustANN(info["dtype"])
    g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), True)
    try:
        nns, _, _, _ = g.hop_search(q.astype(np.uint8).astype(np.float32), 10, 40, index_file=p["index_file"])
    finally:
        g.close()
    formats.write_vecs(str(gf), nns.astype(np.int32))
    cli = os.path.join(ROOT, "gustann_b200", "_lib", "search_mem")
    base = [cli, "--query", str(qf), "--index", p["index_file"], "--pq_data", p["pq_file_prefix"], "--nav_graph",
            p["nav_graph_prefix"], "--ground_truth", str(gf), "--data_type", "uint8", "--topk", "10",
            "--ef_search", "40", "-R", "1"]
    a = subprocess.run(base + ["-G"], capture_output=True, text=True, timeout=300)
    b = subprocess.run(base + ["--hybrid", "-B", "32", "-T", "2"], capture_output=True, text=True, timeout=300)
    # three mini-batches in flight (page reads of one overlap another's hop):
    # 4 batches of 32, 32, 32 and 4 queries, so a slot takes a second batch
    c = subprocess.run(base + ["--hybrid", "-B", "32", "-T", "2", "-C", "3"], capture_output=True, text=True,
                       timeout=300)
    assert a.returncode == 0, a.stderr
    for r in (b, c):
        assert r.returncode == 0, r.stderr
        rec = [float(ln.split()[-1]) for ln in r.stdout.splitlines() if ln.startswith("[REPORT] RECALL:")]
        assert rec and abs(rec[-1] - 1.0) < 1e-9, r.stdout


@pytest.mark.gpu
def test_cli_output_and_check_recall(index_root, tmp_path):
    """search_mem --output writes the bin result file that check_recall
    (bin/check_recall.cpp) scores; both report the same recall against an
    exact ground truth made on the GPU (gann_exact_knn)."""
    import torch
    from gustann_b200 import build as nb
    from gustann_b200.api import exact_knn
    info = get_index(index_root, "u8")
    p = info["paths"]
    q = info["queries"][:200].astype(np.uint8)
    qf, gf, of = tmp_path / "q.bvecs", tmp_path / "gt.ivecs", tmp_path / "out.bin"
    formats.write_vecs(str(qf), q)
    _, X, _, _ = formats.read_disk_index(p["index_file"], formats.UINT8)
    ids, _ = exact_knn(torch.from_numpy(np.ascontiguousarray(X)).cuda(), torch.from_numpy(q).cuda(), 10)
    formats.write_vecs(str(gf), ids.cpu().numpy())
    cli = os.path.join(ROOT, "gustann_b200", "_lib", "search_mem")
    r = subprocess.run([cli, "--query", str(qf), "--index", p["index_file"], "--pq_data", p["pq_file_prefix"],
                        "--nav_graph", p["nav_graph_prefix"], "--ground_truth", str(gf), "--data_type", "uint8",
                        "--topk", "10", "--ef_search", "40", "-R", "1", "-G", "--output", str(of)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rec = [float(ln.split()[-1]) for ln in r.stdout.splitlines() if ln.startswith("[REPORT] RECALL:")]
    c = subprocess.run([nb.build_check(), str(of), str(gf)], capture_output=True, text=True)
    assert c.returncode == 0, c.stdout + c.stderr
    assert rec and c.stdout.strip() == f"Recall @ 10: {rec[-1]:.6f}" and rec[-1] > 0.5
