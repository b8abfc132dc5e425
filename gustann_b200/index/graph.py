"""Graph construction for the disk index and the pivot ("nav") graph.

DiskANN's builder is not available (empty submodule), so the graph is built
here from the published ideas rather than from its code:

1. candidates: exact k nearest neighbours (tiled brute force), or, for large N,
   an IVF partition (k-means lists, each list searched against its ``nprobe``
   nearest lists);
2. long-range candidates: each point's nearest members of progressively coarser
   random samples, which gives the flat graph the "express" edges a hierarchy
   would provide (the pivot-graph greedy search starts from one fixed node);
3. RobustPrune with ``alpha`` on squared L2 (Subramanya et al., NeurIPS 2019):
   walk candidates nearest-first, keep one, drop every later candidate ``c`` with
   ``alpha * d(kept, c) <= d(p, c)``;
4. reverse edges: each kept edge ``p -> q`` offers ``q -> p``; a node whose union
   exceeds ``R`` is pruned again.

Everything is batched torch, so the same code builds tiny test indexes on the
CPU and 10M-point indexes on a GPU.
"""
from __future__ import annotations

import math

import torch


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x if x.dtype == torch.float32 else x.to(torch.float32)


def sq_dists(a: torch.Tensor, b: torch.Tensor, an=None, bn=None) -> torch.Tensor:
    """Squared L2 between rows of ``a`` [m,d] and ``b`` [n,d] (float32)."""
    a = _f32(a)
    b = _f32(b)
    an = (a * a).sum(1) if an is None else an
    bn = (b * b).sum(1) if bn is None else bn
    d = an[:, None] + bn[None, :] - 2.0 * (a @ b.T)
    return d.clamp_min_(0.0)


def knn_exact(X: torch.Tensor, Q: torch.Tensor, k: int, self_offset: int | None = None,
              qblock: int = 2048, xblock: int = 1 << 18):
    """Exact ``k`` nearest rows of ``X`` for every row of ``Q`` (squared L2).

    ``self_offset`` = index in ``X`` of ``Q[0]`` when ``Q`` is a slice of ``X``, so a
    point never lists itself. Returns (ids int64 [nq,k], dist float32 [nq,k]).
    """
    n = X.shape[0]
    k = min(k, n - (1 if self_offset is not None else 0))
    xn = (_f32(X) ** 2).sum(1)
    out_i, out_d = [], []
    for qs in range(0, Q.shape[0], qblock):
        q = _f32(Q[qs: qs + qblock])
        qn = (q * q).sum(1)
        best_d = torch.full((q.shape[0], k), float("inf"), device=X.device)
        best_i = torch.full((q.shape[0], k), -1, dtype=torch.int64, device=X.device)
        for xs in range(0, n, xblock):
            xb = X[xs: xs + xblock]
            d = sq_dists(q, xb, qn, xn[xs: xs + xblock])
            if self_offset is not None:
                rows = torch.arange(q.shape[0], device=X.device)
                cols = rows + self_offset + qs - xs
                ok = (cols >= 0) & (cols < xb.shape[0])
                d[rows[ok], cols[ok]] = float("inf")
            kk = min(k, d.shape[1])
            dv, di = torch.topk(d, kk, dim=1, largest=False)
            cd = torch.cat([best_d, dv], 1)
            ci = torch.cat([best_i, di + xs], 1)
            best_d, sel = torch.topk(cd, k, dim=1, largest=False)
            best_i = torch.gather(ci, 1, sel)
        out_i.append(best_i)
        out_d.append(best_d)
    return torch.cat(out_i), torch.cat(out_d)


def kmeans(X: torch.Tensor, k: int, iters: int, gen: torch.Generator, sample: int = 1 << 18):
    """Lloyd's k-means on a random sample; empty clusters are re-seeded."""
    n = X.shape[0]
    idx = torch.randperm(n, generator=gen, device=X.device)[: min(n, sample)]
    S = _f32(X[idx])
    C = S[torch.randperm(S.shape[0], generator=gen, device=X.device)[:k]].clone()
    for _ in range(iters):
        a = assign(S, C)
        sums = torch.zeros_like(C).index_add_(0, a, S)
        cnt = torch.bincount(a, minlength=C.shape[0]).to(torch.float32)
        empty = cnt == 0
        C = torch.where(empty[:, None], C, sums / cnt.clamp_min(1)[:, None])
        if empty.any():
            ne = int(empty.sum())
            C[empty] = S[torch.randint(0, S.shape[0], (ne,), generator=gen, device=X.device)]
    return C


def assign(X: torch.Tensor, C: torch.Tensor, block: int = 1 << 16) -> torch.Tensor:
    cn = (C * C).sum(1)
    out = []
    for s in range(0, X.shape[0], block):
        out.append(sq_dists(X[s: s + block], C, None, cn).argmin(1))
    return torch.cat(out)


def knn_ivf(X: torch.Tensor, k: int, gen: torch.Generator, nlist: int | None = None,
            nprobe: int = 8, iters: int = 8):
    """Approximate kNN: every point is searched against the members of the
    ``nprobe`` lists whose centroids are nearest to its own list's centroid."""
    n = X.shape[0]
    nlist = nlist or max(16, int(math.sqrt(n)))
    C = kmeans(X, nlist, iters, gen)
    lab = assign(X, C)
    order = torch.argsort(lab)
    counts = torch.bincount(lab, minlength=nlist)
    starts = torch.cumsum(counts, 0) - counts
    near = knn_exact(C, C, min(nprobe, nlist))[0]          # excludes nothing: own list first
    ids = torch.full((n, k), -1, dtype=torch.int64, device=X.device)
    dst = torch.full((n, k), float("inf"), device=X.device)
    counts_l = counts.tolist()
    starts_l = starts.tolist()
    for c in range(nlist):
        if counts_l[c] == 0:
            continue
        mem = order[starts_l[c]: starts_l[c] + counts_l[c]]
        lists = near[c].tolist()
        if c not in lists:
            lists = [c] + lists[:-1]
        cand = torch.cat([order[starts_l[j]: starts_l[j] + counts_l[j]] for j in lists])
        d = sq_dists(X[mem], X[cand])
        d[mem[:, None] == cand[None, :]] = float("inf")
        kk = min(k, cand.shape[0] - 1)
        dv, di = torch.topk(d, kk, dim=1, largest=False)
        ids[mem, :kk] = cand[di]
        dst[mem, :kk] = dv
    return ids, dst


def robust_prune(X: torch.Tensor, p_ids: torch.Tensor, cand: torch.Tensor, cand_d: torch.Tensor,
                 R: int, alpha: float, batch: int = 1 << 14, return_dist: bool = False):
    """RobustPrune for many points at once.

    ``cand`` [B,K] candidate ids sorted nearest-first (-1 = empty), ``cand_d`` their
    squared distances to ``p``. Returns [B,R] kept ids (-1 padded), nearest-first
    (and their distances when ``return_dist``).
    """
    out, outd = [], []
    for s in range(0, cand.shape[0], batch):
        ci = cand[s: s + batch]
        cd = cand_d[s: s + batch]
        b, k = ci.shape
        V = _f32(X[ci.clamp_min(0)])                         # [b,k,d]
        vn = (V * V).sum(-1)
        P = (vn[:, :, None] + vn[:, None, :] - 2.0 * torch.bmm(V, V.transpose(1, 2))).clamp_min_(0)
        alive = ci >= 0
        alive &= ci != p_ids[s: s + batch, None]
        keep = torch.zeros_like(alive)
        count = torch.zeros(b, dtype=torch.int32, device=X.device)
        for j in range(k):
            sel = alive[:, j] & (count < R)
            if not bool(sel.any()):
                if not bool(alive[:, j:].any()):
                    break
                continue
            keep[:, j] = sel
            count += sel.to(torch.int32)
            kill = sel[:, None] & (alpha * P[:, j, :] <= cd)
            alive &= ~kill
        # compact kept ids to the front, preserving nearest-first order
        pos = torch.cumsum(keep.to(torch.int64), 1) - 1
        res = torch.full((b, R), -1, dtype=torch.int64, device=X.device)
        rows = torch.arange(b, device=X.device)[:, None].expand_as(ci)
        m = keep & (pos < R)
        res[rows[m], pos[m]] = ci[m]
        out.append(res)
        if return_dist:
            rd = torch.full((b, R), float("inf"), device=X.device)
            rd[rows[m], pos[m]] = cd[m]
            outd.append(rd)
    if return_dist:
        return torch.cat(out), torch.cat(outd)
    return torch.cat(out)


def _dedup_sorted_rows(ids: torch.Tensor, d: torch.Tensor):
    """Sort each row by (distance, id) and blank out repeated ids."""
    big = torch.where(ids >= 0, d, torch.full_like(d, float("inf")))
    o = torch.argsort(ids, dim=1, stable=True)
    ids_s = torch.gather(ids, 1, o)
    dup = torch.zeros_like(ids_s, dtype=torch.bool)
    dup[:, 1:] = (ids_s[:, 1:] == ids_s[:, :-1]) & (ids_s[:, 1:] >= 0)
    dup_orig = torch.zeros_like(dup).scatter_(1, o, dup)
    big = torch.where(dup_orig, torch.full_like(big, float("inf")), big)
    ids = torch.where(dup_orig, torch.full_like(ids, -1), ids)
    o2 = torch.argsort(big, dim=1, stable=True)
    return torch.gather(ids, 1, o2), torch.gather(big, 1, o2)


def long_range_candidates(X: torch.Tensor, gen: torch.Generator, per_level: int,
                          ratio: int = 16, min_size: int = 64):
    """Each point's ``per_level`` nearest members of nested random samples of size
    n/ratio, n/ratio^2, ... (down to ``min_size``). Returns ([n,c] ids, [n,c] d)."""
    n = X.shape[0]
    perm = torch.randperm(n, generator=gen, device=X.device)
    ids_l, d_l = [], []
    size = n // ratio
    while size >= min_size:
        samp = perm[:size]
        i, d = knn_exact(X[samp], X, per_level)
        ids_l.append(samp[i])
        d_l.append(d)
        size //= ratio
    if not ids_l:
        e = torch.empty(n, 0, device=X.device)
        return e.to(torch.int64), e
    return torch.cat(ids_l, 1), torch.cat(d_l, 1)


def reachable(adj: torch.Tensor, entry: int, block: int = 1 << 22) -> torch.Tensor:
    """Boolean mask of nodes reachable from ``entry`` along out-edges
    (breadth-first; each level marks its neighbours with a scatter, so no sort
    of the frontier is needed at any size)."""
    n = adj.shape[0]
    seen = torch.zeros(n, dtype=torch.bool, device=adj.device)
    mark = torch.zeros(n, dtype=torch.bool, device=adj.device)
    frontier = torch.tensor([entry], device=adj.device, dtype=torch.int64)
    seen[frontier] = True
    while frontier.numel():
        mark.zero_()
        for s in range(0, frontier.numel(), block):
            nb = adj[frontier[s: s + block]].reshape(-1).to(torch.int64)
            mark[nb[nb >= 0]] = True
        mark &= ~seen
        seen |= mark
        frontier = torch.nonzero(mark).reshape(-1)
    return seen


def repair_connectivity(X: torch.Tensor, adj: torch.Tensor, entry: int, rounds: int = 64,
                        inplace: bool = False) -> torch.Tensor:
    """Give every node a path from ``entry``: an unreachable node gets an edge
    from its nearest reachable node, written into that node's free slot or, if
    it has none, over its last (farthest) edge. Repeats until all are reached.
    ``adj`` keeps its dtype; ``inplace`` edits it instead of a copy."""
    adj = adj if inplace else adj.clone()
    n, R = adj.shape
    for _ in range(rounds):
        seen = reachable(adj, entry)
        if bool(seen.all()):
            break
        un = torch.nonzero(~seen).reshape(-1)
        rs = torch.nonzero(seen).reshape(-1)
        Xr, Xu = X[rs], X[un]
        if X.is_cuda and X.dtype in (torch.uint8, torch.float32) and (X.shape[1] * X.element_size()) % 16 == 0:
            from ..api import exact_knn
            near = exact_knn(Xr, Xu, 1)[0].long()
        else:
            near, _ = knn_exact(Xr, Xu, 1)
        del Xr, Xu
        attach_edges(adj, R, rs[near[:, 0]], un)
    return adj


def attach_edges(adj: torch.Tensor, R: int, src: torch.Tensor, dst: torch.Tensor) -> None:
    """Give node src[i] an edge to dst[i], in its first free slot or, if it has
    none, over its last (farthest) edge; one new edge per source node per call
    (the first listed), which keeps each replacement local. An edge a row
    already holds is not added again (a node listed as unreachable can have
    become reachable since, through edges attached earlier in the same round)."""
    ok = src >= 0
    src, dst = src[ok], dst[ok]
    fresh = ~(adj[src, :R] == dst[:, None].to(adj.dtype)).any(1)
    src, dst = src[fresh], dst[fresh]
    order = torch.argsort(src, stable=True)
    src, dst = src[order], dst[order]
    first = torch.ones_like(src, dtype=torch.bool)
    first[1:] = src[1:] != src[:-1]
    src, dst = src[first], dst[first]
    deg = (adj[src, :R] >= 0).sum(1)
    slot = torch.where(deg < R, deg, torch.full_like(deg, R - 1))
    adj[src, slot] = dst.to(adj.dtype)


def build_graph(X: torch.Tensor, R: int, alpha: float = 1.2, k: int | None = None,
                seed: int = 0, long_range: int = 4, exact_limit: int = 300_000,
                nprobe: int = 8, batch: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Build an out-degree <= R graph over ``X``. Returns (adj [n,R] int32 -1-padded,
    deg [n] int32).

    Slots: up to ``R - L - 1`` pruned near neighbours (kNN candidates plus reverse
    edges), up to ``L = min(long_range, R // 4)`` pruned long-range edges kept
    through the reverse-edge step, and one spare slot used by the connectivity
    repair from the medoid.
    """
    n = X.shape[0]
    gen = torch.Generator(device=X.device)
    gen.manual_seed(seed)
    batch = batch or (1 << 16 if X.is_cuda else 1 << 12)
    k = min(k or 2 * R, n - 1)
    n_long = min(long_range, R // 4) if (long_range > 0 and n > 64) else 0
    r_main = max(1, R - n_long - 1)
    if n <= exact_limit:
        ci, cd = knn_exact(X, X, k, self_offset=0)
    else:
        ci, cd = knn_ivf(X, k, gen, nprobe=nprobe)
    pid = torch.arange(n, device=X.device)
    fwd = robust_prune(X, pid, ci, cd, r_main, alpha, batch=batch)
    longe = torch.full((n, 0), -1, dtype=torch.int64, device=X.device)
    if n_long:
        li, ld = long_range_candidates(X, gen, max(long_range, 2))
        li, ld = _dedup_sorted_rows(li, ld)
        longe = robust_prune(X, pid, li, ld, n_long, alpha, batch=batch)

    # reverse edges: q gets p for every kept near edge p -> q, closest R offers only
    src = pid[:, None].expand_as(fwd).reshape(-1)
    dst = fwd.reshape(-1)
    m = dst >= 0
    src, dst = src[m], dst[m]
    rd = ((_f32(X[src]) - _f32(X[dst])) ** 2).sum(1)
    o = torch.argsort(rd, stable=True)
    src, dst, rd = src[o], dst[o], rd[o]
    o = torch.argsort(dst, stable=True)
    src, dst, rd = src[o], dst[o], rd[o]
    cnt = torch.bincount(dst, minlength=n)
    first = torch.cumsum(cnt, 0) - cnt
    rank = torch.arange(dst.shape[0], device=X.device) - first[dst]
    m = rank < R
    rev = torch.full((n, R), -1, dtype=torch.int64, device=X.device)
    revd = torch.full((n, R), float("inf"), device=X.device)
    rev[dst[m], rank[m]] = src[m]
    revd[dst[m], rank[m]] = rd[m]

    fd = torch.where(fwd >= 0, ((_f32(X[fwd.clamp_min(0)]) - _f32(X)[:, None, :]) ** 2).sum(-1),
                     torch.full(fwd.shape, float("inf"), device=X.device))
    ui, ud = _dedup_sorted_rows(torch.cat([fwd, rev], 1), torch.cat([fd, revd], 1))
    # a near candidate that is already a long edge is dropped from the near list
    if n_long:
        dup = (ui[:, :, None] == longe[:, None, :]).any(-1) & (ui >= 0)
        ui = torch.where(dup, torch.full_like(ui, -1), ui)
        ud = torch.where(dup, torch.full_like(ud, float("inf")), ud)
        o = torch.argsort(ud, dim=1, stable=True)
        ui, ud = torch.gather(ui, 1, o), torch.gather(ud, 1, o)
    total = (ui >= 0).sum(1)
    near = ui[:, :r_main].clone()
    over = total > r_main
    if bool(over.any()):
        rows = torch.nonzero(over).reshape(-1)
        near[rows] = robust_prune(X, rows, ui[rows], ud[rows], r_main, alpha, batch=batch)
    parts = [near, longe]
    adj = torch.cat(parts + [torch.full((n, R - r_main - longe.shape[1]), -1, dtype=torch.int64,
                                         device=X.device)], 1)
    # compact each row: valid ids first, order kept
    key = (adj < 0).to(torch.int8)
    o = torch.argsort(key, dim=1, stable=True)
    adj = torch.gather(adj, 1, o)
    deg = (adj >= 0).sum(1)
    lonely = deg == 0
    if bool(lonely.any()):
        adj[lonely, 0] = ci[lonely, 0]
    adj = repair_connectivity(X, adj, medoid(X))
    deg = (adj >= 0).sum(1).to(torch.int32)
    return adj.to(torch.int32), deg


def medoid(X: torch.Tensor) -> int:
    """Index of the point nearest to the mean (the search's default entry)."""
    mu = _f32(X).mean(0, keepdim=True)
    best_d, best_i = float("inf"), 0
    for s in range(0, X.shape[0], 1 << 18):
        d = sq_dists(X[s: s + (1 << 18)], mu).reshape(-1)
        v, i = d.min(0)
        if float(v) < best_d:
            best_d, best_i = float(v), s + int(i)
    return best_i
