"""Product-quantisation training and encoding (256 centroids per chunk).

The layout matches what the search path reads (``src/pq_search.cu:56-121``):
vectors are centred on their mean (``centroid``), split into ``M`` contiguous
chunks given by ``chunk_offsets``, and each chunk of each point is replaced by
the index of its nearest chunk centroid. ``pivots[j]`` concatenates centroid
``j`` of every chunk.
"""
from __future__ import annotations

import numpy as np
import torch

from ..formats import NUM_PIVOTS, chunk_offsets_for
from .graph import _f32, assign


def train_pq(X: torch.Tensor, m: int, seed: int = 0, sample: int = 1 << 18, iters: int = 12):
    """Return (pivots [256,D] f32, centroid [D] f32, chunk_offsets [M+1] u32) as numpy."""
    n, d = X.shape
    gen = torch.Generator(device=X.device)
    gen.manual_seed(seed)
    idx = torch.randperm(n, generator=gen, device=X.device)[: min(n, sample)]
    S = _f32(X[idx])
    centroid = _f32(X).mean(0) if n <= (1 << 22) else S.mean(0)
    S = S - centroid
    offs = chunk_offsets_for(d, m)
    pivots = torch.zeros(NUM_PIVOTS, d, device=X.device)
    for c in range(m):
        a, b = int(offs[c]), int(offs[c + 1])
        sub = S[:, a:b].contiguous()
        if sub.shape[0] >= NUM_PIVOTS:
            C = sub[torch.randperm(sub.shape[0], generator=gen, device=X.device)[:NUM_PIVOTS]].clone()
        else:
            C = sub[torch.randint(0, sub.shape[0], (NUM_PIVOTS,), generator=gen, device=X.device)].clone()
        for _ in range(iters):
            lab = assign(sub, C)
            sums = torch.zeros_like(C).index_add_(0, lab, sub)
            cnt = torch.bincount(lab, minlength=NUM_PIVOTS).to(torch.float32)
            C = torch.where((cnt > 0)[:, None], sums / cnt.clamp_min(1)[:, None], C)
        pivots[:, a:b] = C
    return pivots.cpu().numpy(), centroid.cpu().numpy().astype(np.float32), offs


def encode_pq(X: torch.Tensor, pivots: np.ndarray, centroid: np.ndarray, offs: np.ndarray,
              block: int = 1 << 18) -> np.ndarray:
    """Nearest chunk centroid per chunk of every row; returns [N,M] uint8."""
    dev = X.device
    P = torch.from_numpy(pivots).to(dev)
    cen = torch.from_numpy(centroid).to(dev)
    m = len(offs) - 1
    out = np.empty((X.shape[0], m), dtype=np.uint8)
    for s in range(0, X.shape[0], block):
        R = _f32(X[s: s + block]) - cen
        codes = torch.empty(R.shape[0], m, dtype=torch.uint8, device=dev)
        for c in range(m):
            a, b = int(offs[c]), int(offs[c + 1])
            codes[:, c] = assign(R[:, a:b].contiguous(), P[:, a:b].contiguous()).to(torch.uint8)
        out[s: s + R.shape[0]] = codes.cpu().numpy()
    return out
