"""Why the ADC tables are not built on tensor cores.

A tensor-core table (tcgen05 kind::tf32, the usual three-pass split of each
fp32 operand into a TF32 high part and a TF32 remainder, fp32 accumulation)
computes an entry through the norm expansion |q_b|^2 + |p_bj|^2 - 2 q_b . p_bj,
because (q - p)^2 is not a bilinear form. This test replays those numerics on
the CPU -- TF32 operands (10 explicit mantissa bits, rounded to nearest), exact
TF32 x TF32 products, fp32 sums -- against the oracle's tables (the reference's
fma sequence), then replays the best-first search with both tables on the
committed golden indexes. The split gives products to ~2^-22, but the
expansion cancels: about one entry in 1-2 thousand lands outside the 1e-5
relative tolerance the tables may differ by (up to ~4e-4). On these small
indexes the 48 queries still expanded the same nodes, but nothing bounds that
in general -- one reordered pair of candidates changes the traversal -- while
the kernel's own tables are bit-identical, and the table build is a few
percent of the search. The printed line gives the figures.
"""
import os

import numpy as np
import pytest

from gustann_b200 import formats
from kernel_model import adc_sums, reference_expansions
from oracle import Oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = {"g_u8": formats.UINT8, "g_f32": formats.FLOAT}


def _tf32(x: np.ndarray) -> np.ndarray:
    """Round fp32 to TF32 (10 explicit mantissa bits), to nearest, ties away."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x1000) & 0xFFFFE000
    return b.astype(np.uint32).view(np.float32)


def tf32x3_dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """a [n, k] . b [m, k] with three TF32 passes (hi*hi + hi*lo + lo*hi),
    products exact, sums in fp32 in k order."""
    ah = _tf32(a)
    al = _tf32((a - ah).astype(np.float32))
    bh = _tf32(b)
    bl = _tf32((b - bh).astype(np.float32))
    acc = np.zeros((a.shape[0], b.shape[0]), np.float32)
    for k in range(a.shape[1]):
        for x, y in ((ah, bh), (ah, bl), (al, bh)):
            acc = (acc + np.float32(1) * (x[:, k, None].astype(np.float32) * y[None, :, k].astype(np.float32))).astype(
                np.float32)
    return acc


def tensor_core_lut(q: np.ndarray, piv: np.ndarray, cen: np.ndarray, offs: np.ndarray) -> np.ndarray:
    """[nq, M, 256] entries |q_b|^2 + |p_bj|^2 - 2 q_b . p_bj on q - c."""
    r = (q.astype(np.float32) - cen.astype(np.float32)).astype(np.float32)
    m = len(offs) - 1
    out = np.zeros((q.shape[0], m, 256), np.float32)
    for c in range(m):
        a, b = int(offs[c]), int(offs[c + 1])
        qb, pb = r[:, a:b], piv[:, a:b].astype(np.float32)
        qn = (qb * qb).sum(1, dtype=np.float32)
        pn = (pb * pb).sum(1, dtype=np.float32)
        out[:, c, :] = (qn[:, None] + pn[None, :] - np.float32(2) * tf32x3_dot(qb, pb)).astype(np.float32)
    return out


def _topk(expanded, q, vec, k=10):
    d = ((vec[expanded].astype(np.float64) - q.astype(np.float64)) ** 2).sum(1)
    order = np.argsort(d, kind="stable")
    return [expanded[i] for i in order[:k]]


@pytest.mark.parametrize("name", list(GOLD))
def test_tensor_core_tables_are_not_exact(name):
    dt = GOLD[name]
    p = formats.index_paths(os.path.join(ROOT, "tests", "golden", name))
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], dt)
    piv, cen, offs, codes = formats.read_pq(p["pq_file_prefix"])
    _, vec, deg, nbrs = formats.read_disk_index(p["index_file"], dt)
    q = np.load(os.path.join(ROOT, "tests", "golden", name, "queries.npy"))[:48]
    exact = o.lut(q)
    tc = tensor_core_lut(q, piv, cen, offs)
    rel = np.abs(tc.astype(np.float64) - exact) / np.maximum(np.abs(exact.astype(np.float64)), 1e-30)
    frac_ok = float((rel <= 1e-5).mean())
    _, entries, _ = o.nav(q)
    same, seq = {}, {}
    for ef in (64, 168):
        hit = hs = 0
        for t in range(len(q)):
            def nb(u):
                return nbrs[u, : deg[u]].tolist()
            a, _ = reference_expansions(int(entries[t]), nb, lambda ids: adc_sums(exact[t], codes, ids), ef)
            b, _ = reference_expansions(int(entries[t]), nb, lambda ids: adc_sums(tc[t], codes, ids), ef)
            hit += _topk(a, q[t], vec) == _topk(b, q[t], vec)
            hs += a == b
        same[ef] = hit / len(q)
        seq[ef] = hs / len(q)
    print(f"{name}: max rel err {rel.max():.3g}, entries within 1e-5: {frac_ok:.4f}, "
          f"identical expansion sequences at ef 64 / 168: {seq[64]:.3f} / {seq[168]:.3f}, "
          f"identical top-10 ids: {same[64]:.3f} / {same[168]:.3f}")
    # the kernel's tables are bit-identical to the oracle's (test_gpu_parity);
    # the tensor-core formulation is not, beyond the stated tolerance
    assert rel.max() > 1e-5
    assert frac_ok < 1.0
