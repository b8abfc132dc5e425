"""Query sharding across ranks (one process per GPU, index replicated).

Queries are independent, so a batch splits into contiguous per-rank slices
with no exchange during search; every rank searches its slice on its own GPU.
``gather_results`` is the only collective: it assembles the full result on
rank 0 (``torch.distributed.gather``; NCCL on GPUs, gloo on CPUs) when a caller
wants it there -- the search itself never waits on another rank.

The reference is single-GPU (``scripts/setup.sh:4``); this module is the
multi-GPU extension of its ``GustANN::search`` (``src/ssd_search.cu:114-140``).
"""
from __future__ import annotations

from typing import Callable

import numpy as np
import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of ``n`` items owned by ``rank``; sizes differ by <= 1."""
    if not (0 <= rank < world):
        raise ValueError("rank out of range")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def search_shard(queries: np.ndarray, topk: int, ef: int, search: Callable, rank: int, world: int):
    """Run ``search(q_slice, topk, ef) -> (nns, dist, found)`` on this rank's slice."""
    lo, hi = shard_range(len(queries), rank, world)
    nns, dst, found = search(queries[lo:hi], topk, ef)
    return lo, hi, nns, dst, found


def gather_results(n: int, topk: int, lo: int, nns, dst, found, device="cpu"):
    """Assemble all ranks' slices on rank 0; other ranks get ``None``.

    Every rank must call this (it is a collective)."""
    world = dist.get_world_size()
    rank = dist.get_rank()
    cap = -(-n // world)  # ceil
    buf = torch.zeros((cap, 2 * topk + 2), dtype=torch.float64, device=device)
    m = len(found)
    buf[:m, :topk] = torch.as_tensor(np.asarray(nns), dtype=torch.float64)
    buf[:m, topk:2 * topk] = torch.as_tensor(np.asarray(dst), dtype=torch.float64)
    buf[:m, 2 * topk] = torch.as_tensor(np.asarray(found), dtype=torch.float64)
    buf[:m, 2 * topk + 1] = 1.0
    parts = [torch.zeros_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, parts, dst=0)
    if rank != 0:
        return None
    rows = []
    for r, part in enumerate(parts):
        a, b = shard_range(n, r, world)
        rows.append(part[: b - a])
    full = torch.cat(rows).cpu()
    assert bool((full[:, 2 * topk + 1] == 1).all()), "a rank returned fewer rows than its slice"
    return (full[:, :topk].numpy().astype(np.int32), full[:, topk:2 * topk].numpy().astype(np.float32),
            full[:, 2 * topk].numpy().astype(np.int32))


def exchange_parts(handle, rank: int, world: int) -> None:
    """Split records (``init_pure_mem(..., part_count=world, part_index=rank)``):
    give every rank every other rank's record range. Each rank exports its own
    range (``gann_part_export``), the blobs are all-gathered (a collective:
    every rank calls this once, after opening and before its first search), and
    each rank attaches the others (``gann_part_attach``). Ranks must keep their
    handles open while any rank still searches, because the others read their
    ranges through those mappings."""
    blob = handle.export_part()
    blobs = [None] * world
    dist.all_gather_object(blobs, (rank, blob))
    for src, b in blobs:
        if src != rank:
            handle.attach_part(src, b)
