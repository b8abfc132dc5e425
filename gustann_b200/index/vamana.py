"""Vamana graph construction on the GPU, driven by this library's own search.

Vamana (Subramanya et al., NeurIPS 2019) picks each point's out-edges by
RobustPrune over the nodes a greedy search *from the medoid* visits on the way
to that point, and adds reverse edges; the graph is thereby shaped by the very
search that later runs on it, which is what makes single-entry greedy search
navigate. Points are inserted in batches with prefix doubling (batch sizes
1, 2, 4, ... up to a fraction of N; ParlayANN, Manohar et al., PPoPP 2024).

Each batch's greedy searches are one launch of the fused CUDA search kernel
over the graph being built (``gann_open_device`` on tensors this module
mutates between batches): entry = medoid, ``ef = topk = L``, so the kernel
returns the ``L`` nearest expanded nodes with exact distances -- the candidate
set. RobustPrune runs as one CUDA launch per step (``gann_robust_prune``, a
CTA per point); candidate merging and reverse edges are batched torch ops on
the same GPU.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .graph import _f32, attach_edges, medoid, reachable


def _pad_rows(t: torch.Tensor, mult_bytes: int = 16) -> torch.Tensor:
    row = t.shape[1] * t.element_size()
    if row % mult_bytes == 0 and t.is_contiguous():
        return t
    cols = -(-row // mult_bytes) * mult_bytes // t.element_size()
    out = torch.zeros((t.shape[0], cols), dtype=t.dtype, device=t.device)
    out[:, : t.shape[1]] = t
    return out[:, : t.shape[1]]


def vamana_graph(X: torch.Tensor, codes: np.ndarray, pivots: np.ndarray, centroid: np.ndarray,
                 offs: np.ndarray, R: int = 64, L: int = 100, alpha: float = 1.2, passes: int = 2,
                 seed: int = 0, max_frac: float = 0.02, verbose: bool = False, med: int | None = None):
    """Return (adj [n,R] int32 -1-padded, deg [n] int32, medoid) for CUDA tensor ``X``.

    uint8 vectors are widened to float32 only in the rows a step touches, so
    the builder holds no float copy of the base set."""
    from ..api import GustANN

    assert X.is_cuda, "the Vamana builder runs on the GPU"
    dev = X.device
    n = X.shape[0]
    L = max(L, 8)
    vec = _pad_rows(X.contiguous())
    cd_dev = torch.from_numpy(np.ascontiguousarray(codes)).to(dev)
    cd_dev = _pad_rows(cd_dev)
    rs = -(-R // 4) * 4
    adj = torch.full((n, rs), -1, dtype=torch.int32, device=dev)
    adjd = torch.full((n, R), float("inf"), device=dev)
    med = medoid(X) if med is None else med
    g = GustANN.from_device(vec, adj, cd_dev, pivots, centroid, offs, med, R, device=dev.index or 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    alphas = [1.0, alpha] if passes >= 2 else [alpha]
    stream = torch.cuda.current_stream(dev)
    maxb = max(1, int(max_frac * n))

    def prune(rows, ci, cd, a):
        from ..api import robust_prune as gpu_prune
        return gpu_prune(vec, rows, ci[:, :256], cd[:, :256], R, a)

    def merge(ids2, d2):
        from ..api import sort_unique_rows
        return sort_unique_rows(ids2, d2)

    chunk = 1 << 20      # reverse-edge targets merged per step (bounds the temporaries)
    ar = torch.arange(max(L, R), device=dev)

    def insert(ids: torch.Tensor, a: float):
        b = ids.shape[0]
        q = _f32(X[ids]).contiguous()
        nns = torch.empty((b, L), dtype=torch.int32, device=dev)
        dst = torch.empty((b, L), dtype=torch.float32, device=dev)
        fnd = torch.empty(b, dtype=torch.int32, device=dev)
        g.search_device(q.data_ptr(), b, L, L, nns.data_ptr(), dst.data_ptr(), fnd.data_ptr(), 0,
                        stream.cuda_stream)
        valid = ar[None, :L] < fnd[:, None]
        ci = torch.where(valid, nns, torch.full_like(nns, -1))
        cdv = torch.where(valid, dst, torch.full_like(dst, float("inf")))
        ci, cdv = merge(torch.cat([ci, adj[ids, :R]], 1), torch.cat([cdv, adjd[ids]], 1))
        new, newd = prune(ids, ci, cdv, a)
        adj[ids, :R] = new
        adjd[ids] = newd
        # reverse edges: target t is offered p for each kept edge p -> t, its R
        # closest offers are merged with its row, and an overfull row is pruned
        m = new >= 0
        src = ids[:, None].expand_as(new)[m].to(torch.int32)
        tgt = new[m].long()
        td = newd[m]
        o = torch.argsort(td, stable=True)
        src, tgt, td = src[o], tgt[o], td[o]
        o = torch.argsort(tgt, stable=True)
        src, tgt, td = src[o], tgt[o], td[o]
        uq, cnt = torch.unique_consecutive(tgt, return_counts=True)
        first = torch.cumsum(cnt, 0) - cnt
        take = cnt.clamp_max(R)
        last = max(tgt.shape[0] - 1, 0)
        for c0 in range(0, uq.shape[0], chunk):
            u = uq[c0: c0 + chunk]
            pos = (first[c0: c0 + chunk, None] + ar[None, :R]).clamp_max(last)
            ok = ar[None, :R] < take[c0: c0 + chunk, None]
            inc = torch.where(ok, src[pos], torch.full_like(pos, -1, dtype=torch.int32))
            incd = torch.where(ok, td[pos], torch.full_like(pos, float("inf"), dtype=torch.float32))
            ui, ud = merge(torch.cat([adj[u, :R], inc], 1), torch.cat([adjd[u], incd], 1))
            fit = ui[:, R] < 0
            f = u[fit]
            adj[f, :R] = ui[fit, :R]
            adjd[f] = ud[fit, :R]
            over = ~fit
            rows = u[over]
            if rows.numel():
                pi, pd = prune(rows, ui[over], ud[over], a)
                adj[rows, :R] = pi
                adjd[rows] = pd

    t0 = time.time()
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for pi, a in enumerate(alphas):
            perm = torch.randperm(n, generator=gen, device=dev)
            perm = torch.cat([torch.tensor([med], device=dev), perm[perm != med]])
            i, bsz = 0, 1
            while i < n:
                bs = min(bsz, maxb, n - i)
                insert(perm[i: i + bs], a)
                i += bs
                bsz *= 2
            if verbose:
                torch.cuda.synchronize(dev)
                deg = (adj[:, :R] >= 0).sum(1).float()
                print(f"[vamana] pass {pi} alpha={a}: {time.time() - t0:.1f}s, mean degree {float(deg.mean()):.1f}",
                      flush=True)
        # connectivity: a search from the medoid only expands reachable nodes,
        # so its nearest results for an unreachable point are reachable nodes
        # near it; the nearest with a free slot gets an edge to the point (one
        # new edge per node a round; a full row's last edge is replaced only
        # when none of the candidates has room, since that can cut off another
        # node)
        cands = 16
        for rnd in range(64):
            seen = reachable(adj[:, :R], med)
            if bool(seen.all()):
                break
            un = torch.nonzero(~seen).reshape(-1)
            if verbose:
                print(f"[vamana] repair round {rnd}: {un.numel()} unreachable", flush=True)
            for s0 in range(0, un.numel(), maxb):
                u = un[s0: s0 + maxb]
                b = u.shape[0]
                q = _f32(X[u]).contiguous()
                k = min(cands, L)
                nns = torch.empty((b, k), dtype=torch.int32, device=dev)
                dst = torch.empty((b, k), dtype=torch.float32, device=dev)
                fnd = torch.empty(b, dtype=torch.int32, device=dev)
                g.search_device(q.data_ptr(), b, k, L, nns.data_ptr(), dst.data_ptr(), fnd.data_ptr(), 0,
                                stream.cuda_stream)
                c = nns.long()
                valid = ar[None, :k] < fnd[:, None]
                room = valid & ((adj[c.clamp_min(0), :R] >= 0).sum(-1) < R)
                pick = torch.where(room.any(1), room.int().argmax(1), torch.zeros_like(fnd).long())
                src = torch.where(fnd > 0, c.gather(1, pick[:, None])[:, 0], torch.full_like(pick, -1))
                attach_edges(adj, R, src, u)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32
        g.close()
    out = adj[:, :R].contiguous()
    deg = (out >= 0).sum(1).to(torch.int32)
    return out, deg, med
