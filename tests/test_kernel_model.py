"""CPU check of the CUDA traversal's pool mechanics (tests/kernel_model.py)
against a literal model of the reference's merge, and of the reference model
against the oracle's hop counts, on the committed golden indexes."""
import os

import numpy as np
import pytest

from gustann_b200 import formats
from kernel_model import adc_sums, hop_expansions, kernel_expansions, reference_expansions
from oracle import Oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = {"g_u8": formats.UINT8, "g_f32": formats.FLOAT}


def _load(name):
    dt = GOLD[name]
    p = formats.index_paths(os.path.join(ROOT, "tests", "golden", name))
    lay, vec, deg, nbrs = formats.read_disk_index(p["index_file"], dt)
    _, _, _, codes = formats.read_pq(p["pq_file_prefix"])
    q = np.load(os.path.join(ROOT, "tests", "golden", name, "queries.npy"))
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], dt)
    return o, deg, nbrs, codes, q


@pytest.mark.parametrize("name", list(GOLD))
@pytest.mark.parametrize("ef", [10, 33, 64, 200])
@pytest.mark.parametrize("vis_bits,pool_filter", [(None, False), (5, False), (11, False), (None, True), (5, True)])
def test_kernel_mechanics_equal_reference_merge(name, ef, vis_bits, pool_filter):
    o, deg, nbrs, codes, q = _load(name)
    luts = o.lut(q[:24])
    _, entries, _ = o.nav(q[:24])
    _, _, _, hops, flags = o.search(q[:24], 10, ef)
    for t in range(24):
        lut = luts[t]

        def neighbours(u):
            return nbrs[u, : deg[u]].tolist()

        def adc(ids):
            return adc_sums(lut, codes, ids)

        ref, stale = reference_expansions(int(entries[t]), neighbours, adc, ef)
        ker = kernel_expansions(int(entries[t]), neighbours, adc, ef, vis_bits=vis_bits, pool_filter=pool_filter)
        assert ker == ref, f"query {t}: expansions differ"
        assert len(ref) == hops[t]
        assert stale == bool(flags[t] & 2)


@pytest.mark.parametrize("name", list(GOLD))
@pytest.mark.parametrize("ef", [10, 33, 64])
def test_hop_kernel_merge_equals_reference_merge(name, ef):
    """hop_step_kernel's count-based merge expands the reference's sequence."""
    o, deg, nbrs, codes, q = _load(name)
    luts = o.lut(q[:16])
    _, entries, _ = o.nav(q[:16])
    for t in range(16):
        lut = luts[t]

        def neighbours(u):
            return nbrs[u, : deg[u]].tolist()

        def adc(ids):
            return adc_sums(lut, codes, ids)

        ref, stale = reference_expansions(int(entries[t]), neighbours, adc, ef)
        assert hop_expansions(int(entries[t]), neighbours, adc, ef) == ref, f"query {t}"
