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
set. Pruning and reverse-edge merging are batched torch ops on the same GPU.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .graph import _dedup_sorted_rows, _f32, medoid, robust_prune


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
    """Return (adj [n,R] int32 -1-padded, deg [n] int32, medoid) for CUDA tensor ``X``."""
    from ..api import GustANN

    assert X.is_cuda, "the Vamana builder runs on the GPU"
    dev = X.device
    n = X.shape[0]
    L = max(L, 8)
    Xf = _f32(X).contiguous()
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
    prune_batch = 1 << 15

    def insert(ids: torch.Tensor, a: float):
        b = ids.shape[0]
        q = Xf[ids].contiguous()
        nns = torch.empty((b, L), dtype=torch.int32, device=dev)
        dst = torch.empty((b, L), dtype=torch.float32, device=dev)
        fnd = torch.empty(b, dtype=torch.int32, device=dev)
        g.search_device(q.data_ptr(), b, L, L, nns.data_ptr(), dst.data_ptr(), fnd.data_ptr(), 0,
                        stream.cuda_stream)
        valid = torch.arange(L, device=dev)[None, :] < fnd[:, None]
        ci = torch.where(valid, nns.long(), torch.full_like(nns, -1, dtype=torch.int64))
        cdv = torch.where(valid, dst, torch.full_like(dst, float("inf")))
        ci, cdv = _dedup_sorted_rows(torch.cat([ci, adj[ids, :R].long()], 1), torch.cat([cdv, adjd[ids]], 1))
        new, newd = robust_prune(Xf, ids, ci, cdv, R, a, batch=prune_batch, return_dist=True)
        adj[ids, :R] = new.to(torch.int32)
        adjd[ids] = newd
        # reverse edges, closest R offers per target
        m = new >= 0
        src = ids[:, None].expand_as(new)[m]
        tgt = new[m]
        td = newd[m]
        o = torch.argsort(td, stable=True)
        src, tgt, td = src[o], tgt[o], td[o]
        o = torch.argsort(tgt, stable=True)
        src, tgt, td = src[o], tgt[o], td[o]
        uq, cnt = torch.unique_consecutive(tgt, return_counts=True)
        first = torch.cumsum(cnt, 0) - cnt
        grp = torch.repeat_interleave(torch.arange(uq.shape[0], device=dev), cnt)
        rank = torch.arange(tgt.shape[0], device=dev) - first[grp]
        keep = rank < R
        inc = torch.full((uq.shape[0], R), -1, dtype=torch.int64, device=dev)
        incd = torch.full((uq.shape[0], R), float("inf"), device=dev)
        inc[grp[keep], rank[keep]] = src[keep]
        incd[grp[keep], rank[keep]] = td[keep]
        ui, ud = _dedup_sorted_rows(torch.cat([adj[uq, :R].long(), inc], 1), torch.cat([adjd[uq], incd], 1))
        tot = (ui >= 0).sum(1)
        fit = tot <= R
        if bool(fit.any()):
            f = uq[fit]
            adj[f, :R] = ui[fit, :R].to(torch.int32)
            adjd[f] = ud[fit, :R]
        over = ~fit
        if bool(over.any()):
            rows = uq[over]
            pi, pd = robust_prune(Xf, rows, ui[over], ud[over], R, a, batch=prune_batch, return_dist=True)
            adj[rows, :R] = pi.to(torch.int32)
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
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32
        g.close()
    out = adj[:, :R].contiguous()
    deg = (out >= 0).sum(1).to(torch.int32)
    return out, deg, med
