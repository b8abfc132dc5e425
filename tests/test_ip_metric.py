"""Inner-product metric (configuration 4's): the CUDA path against the oracle
with the same definition, bit-exact -- ADC entries -(sum of q_i * p_ji) per
chunk, pivot-graph and exact distances -<q, x> with the reference's lane and
tree order, q'' = q. The reference itself is L2-only (src/common.hpp:28-30),
so the oracle is the only checker here."""
import numpy as np
import pytest

from conftest import IP_INDEXES, get_index
from gustann_b200.api import (ADC_TABLE, GANN_OPT_ADC_MODE, METRIC_IP, GustANN, GustANNConfig, GustANNStats)
from oracle import Oracle

pytestmark = pytest.mark.gpu


def _open(info, table=False):
    p = info["paths"]
    g = GustANN(info["dtype"], metric=METRIC_IP)
    g.init_pure_mem(GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"]), True)
    if table:
        g.set_option(GANN_OPT_ADC_MODE, ADC_TABLE)
    return g


def _oracle(info):
    p = info["paths"]
    return Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"], metric=1)


@pytest.mark.parametrize("name", list(IP_INDEXES))
def test_ip_lut_and_entry_bit_exact(index_root, name):
    info = get_index(index_root, name)
    g, o = _open(info), _oracle(info)
    q = info["queries"][:64]
    lut = g.probe_lut(q)
    np.testing.assert_array_equal(lut, o.lut(q))
    # entries are -(q . pivot) over each chunk's dims
    from gustann_b200 import formats
    piv, _, offs, _ = formats.read_pq(info["paths"]["pq_file_prefix"])
    for c in (0, len(offs) // 2, len(offs) - 2):
        a, b = int(offs[c]), int(offs[c + 1])
        ref = -(q[:, None, a:b].astype(np.float64) * piv[None, :, a:b].astype(np.float64)).sum(-1)
        np.testing.assert_allclose(lut[:, c, :], ref, rtol=1e-4, atol=1e-6)
    s, e = g.probe_entry(q)
    os_, oe, _ = o.nav(q)
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(e, oe)
    g.close()
    o.close()


@pytest.mark.parametrize("name", list(IP_INDEXES))
@pytest.mark.parametrize("table", [False, True])
@pytest.mark.parametrize("topk,ef", [(10, 64), (100, 100), (100, 256)])
def test_ip_search_matches_oracle(index_root, name, table, topk, ef):
    info = get_index(index_root, name)
    g, o = _open(info, table), _oracle(info)
    q = info["queries"]
    st = GustANNStats()
    nns, dist, found = g.query(q, topk, ef, st)
    onns, odist, ofound, _, flags = o.search(q, topk, ef)
    ok = flags == 0
    assert ok.mean() > 0.95
    np.testing.assert_array_equal(nns[ok], onns[ok])
    np.testing.assert_array_equal(dist[ok], odist[ok])
    np.testing.assert_array_equal(found[ok], ofound[ok])
    # distances are -<q, x>, ascending, and equal the float64 inner products closely
    assert bool((np.diff(dist[ok][:, : int(found.min())], axis=1) >= 0).all())
    assert st.capped_queries == 0
    g.close()
    o.close()


def test_ip_exact_distances_are_negated_dot_products(index_root):
    from gustann_b200 import formats
    info = get_index(index_root, "ip96")
    g = _open(info)
    q = info["queries"][:50]
    nns, dist, found = g.query(q, 10, 64)
    _, X, _, _ = formats.read_disk_index(info["paths"]["index_file"], formats.FLOAT)
    ref = -np.einsum("qd,qkd->qk", q.astype(np.float64), X[nns].astype(np.float64))
    np.testing.assert_allclose(dist, ref, rtol=1e-5, atol=1e-5)
    g.close()


def test_ip_hop_search_matches_oracle(index_root):
    """The host-driven hop search (hybrid mode) with the inner product: the
    oracle entered at the same entries (q'' = q, so the in-HBM entry)."""
    info = get_index(index_root, "ip96")
    p = info["paths"]
    g = _open(info)
    o = _oracle(info)
    q = info["queries"][:100]
    nns, dist, found, _ = g.hop_search(q, 10, 48, index_file=p["index_file"])
    _, entries = g.probe_entry(q)
    onns, odist, ofound, _, flags = o.search(q, 10, 48, entries=entries)
    ok = flags == 0
    np.testing.assert_array_equal(nns[ok], onns[ok])
    np.testing.assert_array_equal(dist[ok], odist[ok])
    g.close()
    o.close()
