"""TEST INFRASTRUCTURE: a host-side model of the CUDA traversal's pool mechanics.

`kernel_expansions` mirrors `traverse()` in gustann_b200/csrc/gann_search.cu
step for step at warp-chunk granularity -- 64-bit candidate keys, the
per-query visited-id table and its hash (every evaluated id, never cleared
within a query; absent when the search has no table buffer), optionally a
pool-membership table (an id only while it is in the pool), the "beyond the last entry" and
duplicate drops, ranks by lower bound, the next node chosen before the merge,
the shifts from sorted survivor ranks + high-to-low moves starting at the
smallest survivor rank's chunk, and the first-unvisited lower bound -- so that
changes to those
mechanics can be checked on the CPU against `reference_expansions`, a literal
model of the reference's merge-path / 2L-cut / dedup / first-unvisited step
(src/impl/pure_mem.cuh:314-419). `hop_expansions` models the count-based merge
of hop_step_kernel (the host-driven hop search). All return the sequence of
expanded node ids; the top-k re-rank does not influence it.

ADC values come from the oracle's bit-exact tables, summed in float32 in chunk
order, exactly as both implementations do.
"""
from __future__ import annotations

import numpy as np

WARP = 32
MASK64 = (1 << 64) - 1


def adc_sums(lut: np.ndarray, codes: np.ndarray, ids) -> np.ndarray:
    """Sequential float32 sums of table entries over chunks 0..M-1."""
    out = np.zeros(len(ids), np.float32)
    m = lut.shape[0]
    for t, v in enumerate(ids):
        s = np.float32(0.0)
        for j in range(m):
            s = np.float32(s + lut[j, codes[v, j]])
        out[t] = s
    return out


def ord_f32(d: np.float32) -> int:
    b = int(np.float32(d + np.float32(0.0)).view(np.uint32))
    return (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)


def key_of(d, v) -> int:
    return (ord_f32(d) << 32) | (int(v) << 1) | 1


def reference_expansions(entry, neighbours, adc, L, max_hops=1 << 14):
    """Literal reference step; returns (expanded ids, stale_flag)."""
    pool_id, pool_d = [], []        # pool with visited bit in id (bit 31)
    u = entry
    out = []
    for _ in range(max_hops):
        out.append(u)
        nb = list(neighbours(u))
        dn = adc(nb)
        new = sorted(zip(dn.tolist(), nb), key=lambda t: (np.float32(t[0]), t[1] & 0x7FFFFFFF))
        sz = len(pool_id)
        merged = [None] * (sz + len(new))
        for t, (d, v) in enumerate(new):       # new element: lower_bound in pool (+1 on same id)
            lo, hi = 0, sz
            while lo < hi:
                mid = (lo + hi) // 2
                if pool_d[mid] < d or (pool_d[mid] == d and (pool_id[mid] & 0x7FFFFFFF) < (v & 0x7FFFFFFF)):
                    lo = mid + 1
                else:
                    hi = mid
            if lo != sz and ((pool_id[lo] ^ v) & 0x7FFFFFFF) == 0:
                lo += 1
            merged[lo + t] = (v, d)
        for i in range(sz):                     # pool element: lower_bound in new
            d, v = pool_d[i], pool_id[i]
            lo, hi = 0, len(new)
            while lo < hi:
                mid = (lo + hi) // 2
                nd, nv = new[mid]
                if nd < d or (nd == d and (nv & 0x7FFFFFFF) < (v & 0x7FFFFFFF)):
                    lo = mid + 1
                else:
                    hi = mid
            merged[lo + i] = (v, d)
        s = min(len(merged), 2 * L)
        merged = merged[:s]
        comp, first = [], None
        for i, (v, d) in enumerate(merged):
            if i and ((merged[i - 1][0] ^ v) & 0x7FFFFFFF) == 0:
                continue
            if first is None and not (v & 0x80000000):
                first = len(comp)
            comp.append((v, d))
        fid = s + 1 if first is None else first
        if fid >= L:
            return out, False
        if fid >= len(comp):
            return out, True
        u = comp[fid][0]
        comp[fid] = (u | 0x80000000, comp[fid][1])
        comp = comp[:L]
        pool_id = [c[0] for c in comp]
        pool_d = [c[1] for c in comp]
    return out, False


def kernel_expansions(entry, neighbours, adc, L, max_hops=1 << 14, vis_bits=11, pool_filter=False):
    """Model of the CUDA traverse(); returns the expanded ids. `vis_bits`
    None models a search without the visited-id table."""
    pl = (L + WARP - 1) // WARP
    fbits = 5
    while (1 << fbits) < pl * WARP:
        fbits += 1
    filt = [0xFFFFFFFF] * (1 << fbits)
    vis = [0xFFFFFFFF] * (1 << vis_bits) if vis_bits else None

    def fslot(i):
        return ((i * 0x9E3779B1) & 0xFFFFFFFF) >> (32 - fbits)

    def vslot(i):
        return ((i * 0x9E3779B1) & 0xFFFFFFFF) >> (32 - vis_bits)

    pool: list[int] = []              # sorted keys; bit 0 = unvisited
    pfirst = 0
    u = entry
    out = []
    for _ in range(max_hops):
        out.append(u)
        nb = list(neighbours(u))
        ok = [(not pool_filter or filt[fslot(v)] != v) and (vis is None or vis[vslot(v)] != v) for v in nb]
        ev = [v for v, k in zip(nb, ok) if k]
        dsum = dict(zip(ev, adc(ev).tolist())) if ev else {}
        if vis is not None:
            for v in ev:
                vis[vslot(v)] = v
        # first unvisited from the hint, chunk by chunk
        psize = len(pool)
        ppos = -1
        j = pfirst >> 5
        while WARP * j < psize:
            hits = [i for i in range(WARP * j, min(WARP * (j + 1), psize)) if pool[i] & 1]
            if hits:
                ppos = hits[0]
                break
            j += 1
        pfirst = ppos if ppos >= 0 else psize
        pstar = pool[ppos] if ppos >= 0 else MASK64
        last = (pool[L - 1] >> 1) if psize == L else MASK64
        surv = []
        for v, k in zip(nb, ok):
            if not k:
                continue
            key = key_of(np.float32(dsum[v]), v)
            kk = key >> 1
            if kk >= last:
                continue
            lo, hi = 0, psize
            while lo < hi:
                mid = (lo + hi) >> 1
                if (pool[mid] >> 1) < kk:
                    lo = mid + 1
                else:
                    hi = mid
            if lo < psize and (pool[lo] >> 1) == kk:
                continue
            surv.append((key, lo))
        mk = min((k for k, _ in surv), default=MASK64)
        nxt = min(mk, pstar)
        more = nxt != MASK64
        S = len(surv)
        if S:
            cpos = []
            for si, (k, r) in enumerate(surv):
                less = sum(1 for t, (o, _) in enumerate(surv) if (o >> 1) < (k >> 1) or ((o >> 1) == (k >> 1) and t < si))
                cpos.append(r + less)
            rmin = min(r for _, r in surv)
            j0 = rmin >> 5
            hist = {}
            for _, r in surv:
                hist[r] = hist.get(r, 0) + 1
            newpool = {i: pool[i] for i in range(min(psize, WARP * j0))}   # untouched prefix
            carry = 0
            shift = {}
            for i in range(WARP * j0, psize):
                carry += hist.get(i, 0)
                shift[i] = carry
            for i in range(psize - 1, WARP * j0 - 1, -1):
                v = pool[i]
                if v == nxt:
                    v &= ~1
                dst = i + shift[i]
                if dst < L:
                    newpool[dst] = v
                else:
                    vid = (v & 0xFFFFFFFF) >> 1
                    if filt[fslot(vid)] == vid:
                        filt[fslot(vid)] = 0xFFFFFFFF
            for (k, _), c in zip(surv, cpos):
                if c < L:
                    kk = k & ~1 if k == nxt else k
                    newpool[c] = kk
                    vid = (kk & 0xFFFFFFFF) >> 1
                    filt[fslot(vid)] = vid
            if nxt == pstar and ppos < WARP * j0:
                newpool[ppos] = pstar & ~1
            psize = min(psize + S, L)
            pool = [newpool[i] for i in range(psize)]
            pfirst = min(pfirst, rmin)
        elif more:
            pool[ppos] = pstar & ~1
        if not more:
            return out
        u = (nxt & 0xFFFFFFFF) >> 1
    return out


def hop_expansions(entry, neighbours, adc, L, max_hops=1 << 14):
    """Model of hop_step_kernel (the host-driven hop search, one launch per
    hop): neighbours equal to a pool entry are dropped; the merged pool puts
    pool entry i at i + #(survivors below it) and survivor e at #(survivors
    below it, ties by slot) + #(pool entries below it), keeps the first L, and
    requests its first unvisited entry (none: done). Returns the expanded ids."""
    pool: list[int] = []
    u = entry
    out = []
    for _ in range(max_hops):
        out.append(u)
        nb = list(neighbours(u))
        dn = adc(nb).tolist() if nb else []
        nk = [key_of(np.float32(d), v) for d, v in zip(dn, nb)]
        ps = len(pool)
        pk = [p >> 1 for p in pool]
        for e, k in enumerate(nk):
            kk = k >> 1
            lo = sum(1 for p in pk if p < kk)     # lower bound in the sorted pool
            if lo < ps and pk[lo] == kk:
                nk[e] = None
        surv = [(e, k) for e, k in enumerate(nk) if k is not None]
        nsz = min(ps + len(surv), L)
        mg = [None] * (ps + len(surv))
        for i, p in enumerate(pool):
            below = sum(1 for _, k in surv if (k >> 1) < (p >> 1))
            mg[i + below] = p
        for e, k in surv:
            below = sum(1 for f, o in surv if (o >> 1) < (k >> 1) or ((o >> 1) == (k >> 1) and f < e))
            lo = sum(1 for p in pk if p < (k >> 1))
            mg[below + lo] = k
        mg = mg[:nsz]
        first = next((j for j, k in enumerate(mg) if k & 1), None)
        if first is None:
            return out
        mg[first] &= ~1
        pool = mg
        u = (mg[first] & 0xFFFFFFFF) >> 1
    return out
