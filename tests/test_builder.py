"""Index builder invariants (graph, PQ, pivot sample) and the synthetic data."""
import numpy as np
import pytest
import torch

from gustann_b200 import formats
from gustann_b200.index import datagen
from gustann_b200.index.graph import build_graph, knn_exact, medoid, robust_prune
from gustann_b200.index.pq import encode_pq, train_pq


def test_datagen_deterministic_and_chunk_independent():
    spec = datagen.MixtureSpec("sift", 3000, 16, 5, 20.0)
    a = datagen.base_vectors(spec)
    b = torch.cat([datagen.base_vectors(spec, start=0, count=1000), datagen.base_vectors(spec, start=1000)])
    assert torch.equal(a, b) and a.dtype == torch.uint8
    d = datagen.MixtureSpec("deep", 100, 8, 3, 0.1)
    x = datagen.base_vectors(d)
    assert torch.allclose(x.norm(dim=1), torch.ones(100), atol=1e-5)
    q0 = datagen.query_vectors(d, 10, offset=0)
    q1 = datagen.query_vectors(d, 10, offset=1)
    assert not torch.equal(q0, q1)


def test_zipf_queries():
    t = datagen.MixtureSpec("text", 100, 16, 50, 0.1, zipf=1.1, query_noise=0.05)
    q = datagen.query_vectors(t, 500)
    assert q.shape == (500, 16) and torch.allclose(q.norm(dim=1), torch.ones(500), atol=1e-5)


def test_knn_exact_matches_brute_force():
    g = torch.Generator().manual_seed(0)
    X = torch.randn(500, 12, generator=g)
    ids, d = knn_exact(X, X, 5, self_offset=0, qblock=64, xblock=128)
    full = ((X[:, None] - X[None]) ** 2).sum(-1)
    full.fill_diagonal_(float("inf"))
    ref = full.topk(5, largest=False)
    assert torch.equal(ids, ref.indices)
    assert torch.allclose(d, ref.values, rtol=1e-4, atol=1e-4)


def test_robust_prune_alpha_one_is_rng():
    # three collinear points: p=0, a=1 (near), b=2 (behind a): b is pruned by a
    X = torch.tensor([[0.0, 0.0], [1.0, 0.0], [2.0, 0.0], [0.0, 1.5]])
    cand = torch.tensor([[1, 3, 2]])
    cd = torch.tensor([[1.0, 2.25, 4.0]])
    out = robust_prune(X, torch.tensor([0]), cand, cd, R=3, alpha=1.0)
    assert out.tolist() == [[1, 3, -1]]


@pytest.mark.parametrize("R", [8, 24])
def test_graph_invariants(R):
    spec = datagen.MixtureSpec("deep", 1500, 16, 6, 0.1, center_scale=0.3)
    X = datagen.base_vectors(spec)
    adj, deg = build_graph(X, R, alpha=1.2)
    n = X.shape[0]
    assert adj.shape == (n, R) and int(deg.min()) >= 1 and int(deg.max()) <= R
    m = torch.arange(R)[None, :] < deg[:, None]
    assert torch.all(adj[m] >= 0) and torch.all(adj[m] < n) and torch.all(adj[~m] == -1)
    assert not torch.any(adj == torch.arange(n)[:, None])           # no self loops
    s = adj.sort(1).values
    assert not torch.any((s[:, 1:] == s[:, :-1]) & (s[:, 1:] >= 0))  # no repeated neighbours
    # the graph reaches everything from the medoid
    seen = torch.zeros(n, dtype=torch.bool)
    frontier = torch.tensor([medoid(X)])
    seen[frontier] = True
    while len(frontier):
        nb = adj[frontier].reshape(-1)
        nb = nb[nb >= 0]
        new = nb[~seen[nb]].unique()
        seen[new] = True
        frontier = new
    assert seen.float().mean() > 0.99


def test_pq_train_and_encode():
    spec = datagen.MixtureSpec("sift", 4000, 32, 8, 20.0)
    X = datagen.base_vectors(spec)
    piv, cen, offs = train_pq(X, 8, iters=4)
    assert piv.shape == (256, 32) and cen.shape == (32,) and offs[-1] == 32
    codes = encode_pq(X, piv, cen, offs)
    assert codes.shape == (4000, 8) and codes.dtype == np.uint8
    r = X.float().numpy() - cen
    rec = np.concatenate([piv[codes[:, c], offs[c]:offs[c + 1]] for c in range(8)], axis=1)
    # reconstruction beats the centroid alone by a wide margin
    assert ((r - rec) ** 2).sum() < 0.3 * (r ** 2).sum()
    # every code is the nearest centroid of its chunk
    c = 3
    a, b = offs[c], offs[c + 1]
    d = ((r[:50, None, a:b] - piv[None, :, a:b]) ** 2).sum(-1)
    assert np.array_equal(d.argmin(1), codes[:50, c]) or np.allclose(
        d.min(1), d[np.arange(50), codes[:50, c]], rtol=1e-5)


def test_pivot_sample_sorted_unique():
    from gustann_b200.index.pipeline import sample_pivots
    s = sample_pivots(10000, 1000)
    assert len(np.unique(s)) == 1000 and np.all(np.diff(s) > 0)


def test_attach_edges_never_duplicates():
    """attach_edges: one edge per source, free slot first, never an edge the
    row already holds."""
    import torch
    from gustann_b200.index.graph import attach_edges
    adj = torch.tensor([[1, 2, -1, -1], [0, 2, 3, 4], [0, -1, -1, -1]], dtype=torch.int32)
    attach_edges(adj, 4, torch.tensor([0, 0, 1, 2]), torch.tensor([2, 3, 5, 0]))
    # row 0: 2 already there, so its next offer (3) fills the free slot; row 1
    # is full and takes 5 over its last edge; row 2 already holds 0
    assert adj.tolist() == [[1, 2, 3, -1], [0, 2, 3, 5], [0, -1, -1, -1]]
