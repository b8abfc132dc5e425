"""Parity of the CUDA path (through the C ABI) with the oracle and with the
reference's own kernels, on identical index files and queries.

Bar: integer outputs (ids, found counts, entry points) identical; distances
and ADC tables bit-identical (the kernel issues the reference's fp32
operations in the reference's order, so the tolerance is zero).
"""
import numpy as np
import pytest

from conftest import INDEXES, get_index
from gustann_b200.api import GustANN, GustANNConfig, GustANNError, GustANNStats
from oracle import F_DUPNBR, F_HOPCAP, F_NAVRACE, F_STALE, Oracle, RefGPU

pytestmark = pytest.mark.gpu

EFS = [10, 33, 64, 100, 200, 480, 1000]


def _open(info, use_gpu_mem=True, nav=True):
    p = info["paths"]
    g = GustANN(info["dtype"])
    g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"] if nav else ""),
                    use_gpu_mem)
    return g


def _oracle(info, nav=True):
    p = info["paths"]
    return Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"] if nav else "", info["dtype"])


@pytest.fixture(scope="module", params=["auto", "table", "separate-codes", "filtered", "filtered-separate"])
def handles(index_root, request):
    """Every index opened over the module in five configurations: ADC mode
    auto with the neighbour-code copy, forced per-query table mode, codes read
    from the shared code array, and the filtered mode (8-bit lower bounds,
    exact ADC only where the bound cannot decide) with either code layout --
    where an index does not allow it (more than 32 chunks or wider than 4
    dims), the filtered configurations fall back to auto."""
    from gustann_b200.api import ADC_FILTERED, ADC_TABLE, GANN_OPT_ADC_MODE, GANN_OPT_NEIGHBOUR_CODES
    out = {}
    for name in INDEXES:
        info = get_index(index_root, name)
        g = _open(info)
        if request.param == "table":
            g.set_option(GANN_OPT_ADC_MODE, ADC_TABLE)
        if request.param in ("separate-codes", "filtered-separate"):
            g.set_option(GANN_OPT_NEIGHBOUR_CODES, 0)
        if request.param.startswith("filtered"):
            try:
                g.set_option(GANN_OPT_ADC_MODE, ADC_FILTERED)
            except GustANNError:
                pass
        out[name] = (info, g, _oracle(info))
    yield out
    for _, g, o in out.values():
        g.close()
        o.close()


@pytest.mark.parametrize("name", list(INDEXES))
def test_lut_bit_exact(handles, name):
    info, g, o = handles[name]
    q = info["queries"][:64]
    np.testing.assert_array_equal(g.probe_lut(q), o.lut(q))


@pytest.mark.parametrize("name", [n for n in INDEXES if INDEXES[n][4]])
def test_entry_matches(handles, name):
    info, g, o = handles[name]
    q = info["queries"]
    s, e = g.probe_entry(q)
    os_, oe, of = o.nav(q)
    ok = (of & F_NAVRACE) == 0
    np.testing.assert_array_equal(s[ok], os_[ok])
    np.testing.assert_array_equal(e[ok], oe[ok])


@pytest.mark.parametrize("name", list(INDEXES))
@pytest.mark.parametrize("ef", EFS)
def test_search_matches_oracle(handles, name, ef):
    info, g, o = handles[name]
    q = info["queries"]
    topk = 10
    st = GustANNStats()
    nns, dist, found = g.query(q, topk, ef, st)
    onns, odist, ofound, ohops, oflags = o.search(q, topk, ef)
    assert st.capped_queries == 0
    assert not np.any(oflags & (F_HOPCAP | F_DUPNBR)), "input outside the reference's defined behaviour"
    # F_STALE queries (the reference would expand a slot it never wrote) stop in
    # both the oracle and the kernel, so they are compared too
    ok = (oflags & F_NAVRACE) == 0
    np.testing.assert_array_equal(found[ok], ofound[ok])
    np.testing.assert_array_equal(nns[ok], onns[ok])
    np.testing.assert_array_equal(dist[ok], odist[ok])
    assert st.hops == int(ohops[ok].sum()) or not ok.all()


@pytest.mark.parametrize("name", ["u8", "f32"])
def test_topk_edge_cases(handles, name):
    info, g, o = handles[name]
    q = info["queries"][:100]
    for topk, ef in [(1, 1), (1, 16), (16, 16), (64, 64), (100, 128)]:
        nns, dist, found = g.query(q, topk, ef)
        onns, odist, ofound, _, oflags = o.search(q, topk, ef)
        ok = (oflags & F_NAVRACE) == 0
        np.testing.assert_array_equal(nns[ok], onns[ok])
        np.testing.assert_array_equal(dist[ok], odist[ok])
        np.testing.assert_array_equal(found[ok], ofound[ok])


def test_no_nav_uses_medoid(index_root):
    info = get_index(index_root, "u8")
    g = _open(info, nav=False)
    o = _oracle(info, nav=False)
    q = info["queries"][:200]
    nns, dist, found = g.query(q, 10, 40)
    onns, odist, ofound, _, oflags = o.search(q, 10, 40)
    assert not (oflags & (F_HOPCAP | F_DUPNBR)).any()
    np.testing.assert_array_equal(nns, onns)
    np.testing.assert_array_equal(dist, odist)
    g.close()


def test_host_records_mode_equal(index_root):
    """use_gpu_mem=False keeps records in pinned host memory (the reference's
    search_graph_kernel_dram mode); results are the same."""
    info = get_index(index_root, "f32")
    a = _open(info, use_gpu_mem=True)
    b = _open(info, use_gpu_mem=False)
    q = info["queries"][:200]
    for ef in (20, 80):
        x = a.query(q, 10, ef)
        y = b.query(q, 10, ef)
        for u, v in zip(x, y):
            np.testing.assert_array_equal(u, v)
    a.close()
    b.close()


def test_device_entry_point(index_root):
    import torch
    info = get_index(index_root, "f32")
    g = _open(info)
    q = info["queries"][:300]
    topk, ef = 10, 64
    dq = torch.from_numpy(q).cuda()
    dn = torch.zeros((len(q), topk), dtype=torch.int32, device="cuda")
    dd = torch.zeros((len(q), topk), dtype=torch.float32, device="cuda")
    df = torch.zeros(len(q), dtype=torch.int32, device="cuda")
    dh = torch.zeros(len(q), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()
    g.search_device(dq.data_ptr(), len(q), topk, ef, dn.data_ptr(), dd.data_ptr(), df.data_ptr(), dh.data_ptr(),
                    s.cuda_stream)
    torch.cuda.synchronize()
    nns, dist, found = g.query(q, topk, ef)
    np.testing.assert_array_equal(dn.cpu().numpy(), nns)
    np.testing.assert_array_equal(dd.cpu().numpy(), dist)
    np.testing.assert_array_equal(df.cpu().numpy(), found)
    assert int(dh.sum()) > 0
    g.close()


def test_empty_and_single_query(handles):
    info, g, o = handles["u8"]
    nns, dist, found = g.query(info["queries"][:0], 10, 20)
    assert nns.shape == (0, 10)
    q1 = info["queries"][:1]
    x = g.query(q1, 10, 20)
    y = o.search(q1, 10, 20)
    np.testing.assert_array_equal(x[0], y[0])


def test_bad_arguments_raise(handles):
    info, g, _ = handles["u8"]
    q = info["queries"][:4]
    with pytest.raises(GustANNError):
        g.query(q, 20, 10)          # topk > ef
    with pytest.raises(GustANNError):
        g.query(q, 10, 100000)      # ef beyond the supported maximum


# The reference's own kernels did not finish on the 768-dim, 96-chunk index
# (f32_wide) within the 25 minutes of a test run on a B200, so they are not
# run on that shape again; its parity rests on the oracle, which the
# reference's kernels pin on the other shapes.
REF_SHAPES = [n for n in INDEXES if n != "f32_wide"]


@pytest.mark.skipif(not RefGPU.available(), reason="reference library not built")
@pytest.mark.parametrize("name", REF_SHAPES)
def test_reference_kernels_agree(handles, name):
    """The reference's own compiled kernels on the B200, same files and queries.

    The reference is handed only queries the oracle shows to be inside its
    defined behaviour at that ef (flags == 0): on the others it would expand a
    pool slot it never wrote or index its pivot map out of range, which can
    read outside its buffers. Queries are independent there (one CTA each), so
    dropping them changes nothing for the rest."""
    info, g, o = handles[name]
    p = info["paths"]
    r = RefGPU(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"], info["dim"])
    q = info["queries"][:200]
    np.testing.assert_array_equal(r.lut(q[:32], info["M"]), g.probe_lut(q[:32]))
    if p["nav_graph_prefix"]:
        os_, _, of = o.nav(q)
        s_cnt = len(np.loadtxt(p["nav_graph_prefix"] + "/map.txt", ndmin=1))
        # the reference's nav loop has no iteration bound: queries whose oracle
        # replay hit the hop cap would spin there, so they are never handed over
        clean = ((of & (F_NAVRACE | F_HOPCAP)) == 0) & (os_ >= 0) & (os_ < s_cnt)
        rs, re = r.nav(q[clean])
        s, e = g.probe_entry(q[clean])
        np.testing.assert_array_equal(rs, s)
        np.testing.assert_array_equal(re, e)
    for ef in (10, 64, 200, 700):
        of = o.search(q, 10, ef)[4]
        qc = q[of == 0]              # no hop cap, stale slot, repeated id or nav race
        assert len(qc) > len(q) // 2
        rn, rd, rf, _ = r.search(qc, 10, ef)
        nns, dist, found = g.query(qc, 10, ef)
        np.testing.assert_array_equal(rf, found)
        np.testing.assert_array_equal(rn, nns)
        np.testing.assert_array_equal(rd, dist)
    r.close()


def test_pivot_mode_option(index_root):
    from gustann_b200.api import ADC_PIVOT, ADC_TABLE, GANN_OPT_ADC_MODE, GANN_OPT_PIVOT_WARPS
    info = get_index(index_root, "f32")
    g = _open(info)
    q = info["queries"][:300]
    g.set_option(GANN_OPT_ADC_MODE, ADC_TABLE)
    ref = g.query(q, 10, 48)
    g.set_option(GANN_OPT_ADC_MODE, ADC_PIVOT)
    for w in (8, 13, 20, 0):
        g.set_option(GANN_OPT_PIVOT_WARPS, w)
        out = g.query(q, 10, 48)
        for u, v in zip(ref, out):
            np.testing.assert_array_equal(u, v)
    with pytest.raises(GustANNError):
        g.set_option(GANN_OPT_PIVOT_WARPS, 7)
    g.close()
