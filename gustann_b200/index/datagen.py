"""Seeded synthetic stand-ins for the datasets the reference is measured on.

No SIFT/DEEP/BIGANN files exist on these machines, so every vector set is drawn
from a Gaussian mixture with the shapes of the benchmark configurations:

* ``sift``: centers uniform in ``[0, 128]^D``, per-dimension sigma, rounded and
  clipped to ``[0, 255]`` (uint8 records, SIFT-like).
* ``deep``: centers ``N(0, center_scale^2 I)`` -- or, with ``center_rank`` r, drawn
  on a random r-dimensional subspace with the same per-dimension scale (real
  embedding sets have low intrinsic dimension) -- per-dimension sigma, every
  vector L2-normalised (float32 records, DEEP-like).
* ``text``: as ``deep`` but queries pick their cluster with a Zipf(1.1) law and get
  ``N(0, 0.05^2)`` noise (inner-product configuration).

Generation is chunked and every chunk has its own seed derived from
``(seed, chunk index)``, so any chunk can be regenerated alone and the result does
not depend on the chunk size used by the caller.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

SEED_CENTERS = 0
SEED_DATA = 1
SEED_QUERIES = 2
CHUNK = 1 << 18


@dataclass
class MixtureSpec:
    kind: str                 # "sift" | "deep" | "text"
    n: int
    dim: int
    centers: int
    sigma: float
    center_scale: float = 1.0
    zipf: float | None = None     # queries only (text)
    query_noise: float | None = None
    center_rank: int | None = None  # deep/text: centers span a subspace of this rank
    seeds: dict = field(default_factory=lambda: {
        "centers": SEED_CENTERS, "data": SEED_DATA, "queries": SEED_QUERIES})

    @property
    def dtype(self) -> int:
        return 0 if self.kind == "sift" else 1


# The five configurations of the benchmark description (sizes as stated there).
# deep/text centers are random directions of unit expected norm (per-dimension
# scale 1/sqrt(D)); sigma is per dimension before normalisation.
CONFIGS = {
    "c0": MixtureSpec("sift", 1_000_000, 128, 1000, 20.0),
    "c1": MixtureSpec("deep", 10_000_000, 96, 2000, 0.1, center_scale=96 ** -0.5),
    "c2": MixtureSpec("sift", 100_000_000, 128, 10_000, 20.0),
    "c3": MixtureSpec("sift", 1_000_000_000, 128, 100_000, 20.0),
    "c4": MixtureSpec("text", 10_000_000, 768, 5000, 0.1 * (96 / 768) ** 0.5, center_scale=768 ** -0.5,
                      zipf=1.1, query_noise=0.05),
}


def _gen(device, seed: int, sub: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + sub) & 0x7FFF_FFFF_FFFF_FFFF)
    return g


def centers(spec: MixtureSpec, device="cpu") -> torch.Tensor:
    g = _gen(device, spec.seeds["centers"], 0)
    if spec.kind == "sift":
        return torch.rand(spec.centers, spec.dim, generator=g, device=device) * 128.0
    if spec.center_rank:
        r = spec.center_rank
        z = torch.randn(spec.centers, r, generator=g, device=device)
        a = torch.randn(r, spec.dim, generator=g, device=device)
        return (z @ a) * (spec.center_scale / r ** 0.5)
    return torch.randn(spec.centers, spec.dim, generator=g, device=device) * spec.center_scale


def _finish(spec: MixtureSpec, x: torch.Tensor) -> torch.Tensor:
    if spec.kind == "sift":
        return x.round_().clamp_(0, 255).to(torch.uint8)
    return torch.nn.functional.normalize(x, dim=1)


def _chunk(spec, cen, seed, idx, count, device, zipf=None, noise=None):
    g = _gen(device, seed, idx)
    if zipf is None:
        lab = torch.randint(0, spec.centers, (count,), generator=g, device=device)
    else:
        ranks = torch.arange(1, spec.centers + 1, device=device, dtype=torch.float64)
        p = ranks.pow(-zipf)
        lab = torch.multinomial((p / p.sum()).float(), count, replacement=True, generator=g)
    sig = spec.sigma if noise is None else noise
    x = cen[lab] + sig * torch.randn(count, spec.dim, generator=g, device=device)
    return _finish(spec, x)


def base_vectors(spec: MixtureSpec, device="cpu", start: int = 0, count: int | None = None) -> torch.Tensor:
    """Rows ``[start, start+count)`` of the base set (chunk-seeded, order independent)."""
    count = spec.n - start if count is None else count
    cen = centers(spec, device)
    out = []
    c0, c1 = start // CHUNK, (start + count - 1) // CHUNK
    for c in range(c0, c1 + 1):
        lo = c * CHUNK
        rows = min(CHUNK, spec.n - lo)
        blk = _chunk(spec, cen, spec.seeds["data"], c, rows, device)
        a = max(start, lo) - lo
        b = min(start + count, lo + rows) - lo
        out.append(blk[a:b])
    return torch.cat(out) if out else torch.empty(0, spec.dim, device=device)


def query_vectors(spec: MixtureSpec, nq: int, device="cpu", offset: int = 0) -> torch.Tensor:
    """``nq`` queries; ``offset`` selects a disjoint query stream (one per rank)."""
    cen = centers(spec, device)
    return _chunk(spec, cen, spec.seeds["queries"], 7919 * offset, nq, device,
                  zipf=spec.zipf, noise=spec.query_noise)


def as_float_queries(q: torch.Tensor) -> np.ndarray:
    """Queries as the float32 rows ``search`` takes (u8 queries are widened,
    ``bin/search_disk.cpp:160-165``)."""
    return q.to(torch.float32).cpu().numpy()
