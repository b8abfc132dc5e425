"""Round trips of every on-disk format and the record geometry rules."""
import os

import numpy as np
import pytest

from gustann_b200 import formats


def test_vecs_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    for dt in (np.float32, np.int32, np.uint8):
        a = (rng.random((17, 9)) * 200).astype(dt)
        p = str(tmp_path / f"x.{np.dtype(dt).name}")
        formats.write_vecs(p, a)
        assert np.array_equal(formats.read_vecs(p, dt), a)
        assert os.path.getsize(p) == 17 * (4 + 9 * np.dtype(dt).itemsize)


def test_bad_vecs_size(tmp_path):
    p = str(tmp_path / "bad.fvecs")
    formats.write_vecs(p, np.zeros((3, 4), np.float32))
    with open(p, "ab") as f:
        f.write(b"\0\0")
    with pytest.raises(ValueError):
        formats.read_vecs(p, np.float32)


@pytest.mark.parametrize("dtype,dim,R", [(formats.UINT8, 128, 64), (formats.FLOAT, 96, 64), (formats.FLOAT, 768, 64),
                                         (formats.UINT8, 7, 3)])
def test_disk_index_round_trip(tmp_path, dtype, dim, R):
    rng = np.random.default_rng(1)
    n = 257
    t = formats.np_dtype(dtype)
    vec = (rng.random((n, dim)) * 200).astype(t)
    deg = rng.integers(1, R + 1, n)
    adj = rng.integers(0, n, (n, R))
    p = str(tmp_path / "i.index")
    lay = formats.write_disk_index(p, vec, adj, deg, medoid=5, max_m0=R)
    node_len, npp = formats.record_geometry(dim, np.dtype(t).itemsize, R)
    assert lay.max_node_len == node_len and lay.nodes_per_page == npp
    assert os.path.getsize(p) == (1 + (n + npp - 1) // npp) * 4096
    lay2, vec2, deg2, nb2 = formats.read_disk_index(p, dtype)
    assert lay2 == lay
    assert np.array_equal(vec2, vec) and np.array_equal(deg2, deg)
    m = np.arange(R)[None, :] < deg[:, None]
    assert np.array_equal(nb2[m], adj[m])


def test_record_geometry_of_the_five_configurations():
    # node_len / nodes per page of the five configurations
    assert formats.record_geometry(128, 1, 64) == (388, 10)
    assert formats.record_geometry(96, 4, 64) == (644, 6)
    assert formats.record_geometry(768, 4, 64) == (3332, 1)
    with pytest.raises(ValueError):
        formats.record_geometry(1024, 4, 64)


@pytest.mark.parametrize("legacy", [False, True])
def test_pq_round_trip(tmp_path, legacy):
    rng = np.random.default_rng(2)
    dim, m, n = 96, 32, 100
    piv = rng.random((256, dim)).astype(np.float32)
    cen = rng.random(dim).astype(np.float32)
    offs = formats.chunk_offsets_for(dim, m)
    codes = rng.integers(0, 256, (n, m)).astype(np.uint8)
    pre = str(tmp_path / "pq")
    formats.write_pq(pre, piv, cen, offs, codes, legacy=legacy)
    a, b, c, d = formats.read_pq(pre)
    assert np.array_equal(a, piv) and np.array_equal(b, cen) and np.array_equal(c, offs) and np.array_equal(d, codes)
    tab = formats.read_bin(pre + "_pivots.bin", np.uint64, 0).reshape(-1)
    assert tab[0] == 4096 and len(tab) == (5 if legacy else 4)


def test_chunk_offsets():
    assert list(formats.chunk_offsets_for(128, 32)[:3]) == [0, 4, 8]
    o = formats.chunk_offsets_for(100, 32)          # 4 chunks of 4 dims, 28 of 3
    assert o[-1] == 100 and np.all(np.diff(o) >= 3) and np.diff(o)[0] == 4
    with pytest.raises(ValueError):
        formats.chunk_offsets_for(4, 8)


def test_nav_round_trip(tmp_path):
    rng = np.random.default_rng(3)
    s, dim = 50, 16
    vec = rng.random((s, dim)).astype(np.float32)
    ids = np.sort(rng.choice(1000, s, replace=False)).astype(np.int32)
    deg = rng.integers(1, 33, s)
    adj = rng.integers(0, s, (s, 32)).astype(np.int32)
    formats.write_nav(str(tmp_path / "nav"), vec, ids, adj, deg, start=7, max_degree=32)
    v2, a2, st, i2 = formats.read_nav(str(tmp_path / "nav"), formats.FLOAT)
    assert st == 7 and np.array_equal(v2, vec) and np.array_equal(i2, ids)
    m = np.arange(32)[None, :] < deg[:, None]
    assert np.array_equal(a2[m], adj[m]) and np.all(a2[~m] == -1)
    raw = np.fromfile(str(tmp_path / "nav" / "nav_index"), dtype=np.uint32)
    assert raw[2] == 32 and raw[3] == 7       # max degree at byte 8, start at byte 12
