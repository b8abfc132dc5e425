"""The allocation-free entry point, gann_search_noalloc, called through the C ABI.

It serves callers that cannot call cudaMalloc while searching (their device
memory comes from another runtime's arena, or an allocation's device-wide
synchronisation is not acceptable mid-flight): the index arrays, queries and
outputs are theirs, and the library's own per-call device state lives in a
static device array. Its results must equal those of the existing entry point
(gann_open_device + gann_search_device) over the same arrays, bit for bit, on
consecutive calls -- the second call also proves the shared scratch is reset --
and those of the CPU oracle entered at the same node (the medoid: this
descriptor has no pivot graph).

This file is collected last on purpose, and passes alone or after the others.
"""
import ctypes as C
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

GOLD = {"g_f32": 1, "g_u8": 0}


def _device_index(name):
    import torch
    from gustann_b200 import formats
    p = formats.index_paths(os.path.join(ROOT, "tests", "golden", name))
    dtype = GOLD[name]
    lay, vec, deg, nbrs = formats.read_disk_index(p["index_file"], dtype)
    adj = np.where(np.arange(lay.max_m0)[None, :] < deg[:, None], nbrs.astype(np.int64), -1).astype(np.int32)
    pivots, centroid, offs, codes = formats.read_pq(p["pq_file_prefix"])
    row = -(-vec.shape[1] * vec.itemsize // 16) * 16 // vec.itemsize
    v = np.zeros((vec.shape[0], row), vec.dtype)
    v[:, : vec.shape[1]] = vec
    cs = -(-codes.shape[1] // 16) * 16
    c = np.zeros((codes.shape[0], cs), np.uint8)
    c[:, : codes.shape[1]] = codes
    astr = -(-lay.max_m0 // 4) * 4
    a = np.full((adj.shape[0], astr), -1, np.int32)
    a[:, : adj.shape[1]] = adj
    t = {"vec": torch.from_numpy(v).cuda()[:, : vec.shape[1]], "adj": torch.from_numpy(a).cuda(),
         "codes": torch.from_numpy(c).cuda()}
    q = np.load(os.path.join(ROOT, "tests", "golden", name, "queries.npy"))
    return t, pivots, centroid, offs, lay, q, p


def _descriptor(api, t, pivots, centroid, offs, lay):
    piv = np.ascontiguousarray(pivots, np.float32)
    cen = np.ascontiguousarray(centroid, np.float32)
    off = np.ascontiguousarray(offs, np.uint32)
    vec = t["vec"]
    d = api._DeviceIndex(vec.data_ptr(), vec.stride(0) * vec.element_size(), t["adj"].data_ptr(),
                         t["adj"].stride(0), lay.max_m0, t["codes"].data_ptr(), t["codes"].stride(0),
                         len(off) - 1, piv.ctypes.data_as(C.c_void_p), cen.ctypes.data_as(C.c_void_p),
                         off.ctypes.data_as(C.c_void_p), vec.shape[0], vec.shape[1],
                         0 if vec.element_size() == 1 else 1, lay.medoid, 0)
    return d, (piv, cen, off)


@pytest.mark.parametrize("name", list(GOLD))
def test_noalloc_matches_existing_entry_point(name):
    import torch
    from gustann_b200 import api
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle
    t, pivots, centroid, offs, lay, q, paths = _device_index(name)
    o = Oracle(paths["index_file"], paths["pq_file_prefix"], "", GOLD[name])
    dq = torch.from_numpy(q).cuda()
    nq = len(q)
    stream = torch.cuda.current_stream()
    g = api.GustANN.from_device(t["vec"], t["adj"], t["codes"], pivots, centroid, offs, lay.medoid, lay.max_m0)
    desc, keep = _descriptor(api, t, pivots, centroid, offs, lay)
    try:
        for topk, ef in ((10, 20), (10, 40)):            # two calls in a row
            outs = []
            for which in ("existing", "noalloc"):
                nns = torch.full((nq, topk), -7, dtype=torch.int32, device="cuda")
                dst = torch.full((nq, topk), -7.0, dtype=torch.float32, device="cuda")
                fnd = torch.full((nq,), -7, dtype=torch.int32, device="cuda")
                if which == "existing":
                    g.search_device(dq.data_ptr(), nq, topk, ef, nns.data_ptr(), dst.data_ptr(), fnd.data_ptr(), 0,
                                    stream.cuda_stream)
                else:
                    dev_before = torch.cuda.current_device()
                    rc = api.lib.gann_search_noalloc(C.byref(desc), dq.data_ptr(), nq, topk, ef, nns.data_ptr(),
                                                     dst.data_ptr(), fnd.data_ptr(), stream.cuda_stream)
                    assert rc == api.GANN_OK, api.lib.gann_last_error()
                    assert torch.cuda.current_device() == dev_before
                torch.cuda.synchronize()
                outs.append((nns.cpu().numpy(), dst.cpu().numpy(), fnd.cpu().numpy()))
            for a, b in zip(*outs):
                np.testing.assert_array_equal(a, b)
            assert (outs[1][2] == topk).all()
            onns, odist, ofound, _, flags = o.search(q, topk, ef, entries=np.full(nq, lay.medoid, np.int32))
            ok = flags == 0
            assert ok.mean() > 0.9
            np.testing.assert_array_equal(outs[1][0][ok], onns[ok])
            np.testing.assert_array_equal(outs[1][1][ok], odist[ok])
            np.testing.assert_array_equal(outs[1][2][ok], ofound[ok])
    finally:
        g.close()
        o.close()


def test_noalloc_rejects_oversized_index():
    """An index whose staged tables exceed the static scratch gets a clear error."""
    import torch
    from gustann_b200 import api
    dim, m = 1024, 128
    vec = torch.zeros((8, dim), dtype=torch.float32, device="cuda")
    adj = torch.full((8, 4), -1, dtype=torch.int32, device="cuda")
    codes = torch.zeros((8, 128), dtype=torch.uint8, device="cuda")
    piv = np.zeros((256, dim), np.float32)
    cen = np.zeros(dim, np.float32)
    off = (np.arange(m + 1) * (dim // m)).astype(np.uint32)
    d = api._DeviceIndex(vec.data_ptr(), dim * 4, adj.data_ptr(), 4, 4, codes.data_ptr(), 128, m,
                         piv.ctypes.data_as(C.c_void_p), cen.ctypes.data_as(C.c_void_p),
                         off.ctypes.data_as(C.c_void_p), 8, dim, 1, 0, 0)
    out = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = api.lib.gann_search_noalloc(C.byref(d), vec.data_ptr(), 1, 1, 1, out.data_ptr(), out.data_ptr(),
                                     out.data_ptr(), None)
    assert rc == api.GANN_EUNSUPPORTED
    assert b"static scratch" in api.lib.gann_last_error()
