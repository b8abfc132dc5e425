"""Record order of an index: rows grouped by a coarse partition.

A search hop reads one record and its neighbours' PQ code rows at random
places of the index. Over a 100M-point index (about 42 GB) such reads touch far
more device pages than the GPU's address-translation caches cover, and the
misses lengthen every hop. Storing the rows grouped by a coarse partition
keeps graph neighbours, which are near each other in space, also near each
other in memory, so a query's hops stay within a few pages.

The partition: `parts` rows drawn at random serve as centers and every row
goes to its nearest center (exact L2, ``gann_exact_knn``); rows are ordered by
center, then by input position. The permutation is returned new-to-old: row i
of the reordered set is input row ``perm[i]``.
"""
from __future__ import annotations

import torch


def partition_order(X: torch.Tensor, parts: int = 16384, seed: int = 7, block: int = 1 << 20) -> torch.Tensor:
    """New-to-old int64 permutation of the rows of ``X`` (CUDA, uint8 or
    float32, rows 16-byte aligned) grouping them by nearest sampled center."""
    from ..api import exact_knn
    n = X.shape[0]
    parts = max(1, min(parts, n))
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    pick = torch.randperm(n, generator=g)[:parts].sort().values.to(X.device)
    centers = X[pick].contiguous()
    label = torch.empty(n, dtype=torch.int64, device=X.device)
    for s in range(0, n, block):
        ids, _ = exact_knn(centers, X[s: s + block], 1)
        label[s: s + ids.shape[0]] = ids[:, 0].to(torch.int64)
    # stable: ties (same center) keep input order
    return torch.sort(label, stable=True).indices
