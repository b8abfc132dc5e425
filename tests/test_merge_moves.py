"""The pool merge's move loops of traverse() (gustann_b200/csrc/gann_search.cu),
replayed lane by lane on the CPU.

After a hop, S surviving candidates enter the sorted pool at their ranks (lower
bounds). The kernel moves pool entries right, from the last chunk down, and
touches no entry before the smallest survivor rank: chunks at or after the
largest survivor rank move by S as a whole (phase A); the chunks below take
each entry's own shift, the number of survivor ranks <= its position, found by
power-of-two steps over the sorted ranks, four chunks at a time (phase B).
Entries pushed past ef leave the pool, and the entry equal to the next node is
written back marked visited. The replay must give exactly the first ef keys of
the merged set, for random pools, survivor sets and ef, including survivors
at rank 0, at the end, all at one rank, and more survivors than free slots.
"""
import random

WARP = 32


def kernel_merge(pool, surv, L, nxt, ppos, pstar):
    """Lane-level replay of the kernel's merge; `surv` = [(key, rank)], keys
    sorted by the caller the way the kernel counts `less`."""
    psize, S = len(pool), len(surv)
    buf = list(pool) + [None] * (L - len(pool))
    cr = [r for _, r in surv]
    cpos = []
    for si, (k, r) in enumerate(surv):
        less = sum(1 for t, (o, _) in enumerate(surv) if (o >> 1) < (k >> 1) or ((o >> 1) == (k >> 1) and t < si))
        cpos.append(r + less)
    rmin, rmax = min(cr), max(cr)
    hist = [0] * S
    for (k, r), c in zip(surv, cpos):
        hist[c - r] = r
    j0 = rmin >> 5
    ju = (rmax + WARP - 1) >> 5
    # phase A: whole chunks move by S
    j = min((psize - 1) >> 5, (L - 1 - S) >> 5)
    while j >= ju and j >= j0:
        vals = []
        for lane in range(WARP):
            i = lane + WARP * j
            v = buf[i] if i < psize else 0
            if v == nxt:
                v &= ~1
            vals.append(v)
        for lane in range(WARP):          # __syncwarp between the reads and the writes
            i = lane + WARP * j
            if i < psize and i + S < L:
                buf[i + S] = vals[lane]
        j -= 1
    # phase B: four chunks at a time, each entry's own shift
    sstep = 1 << (S.bit_length() - 1)
    jg = min((psize - 1) >> 5, ju - 1)
    while jg >= j0:
        reads = []
        for g in range(4):
            for lane in range(WARP):
                i = lane + WARP * (jg - g)
                act = jg - g >= j0 and i < psize
                v = buf[i] if act else 0
                sh = 0
                step = sstep
                while step > 0:
                    t = sh + step
                    if act and t <= S and hist[t - 1] <= i:
                        sh = t
                    step >>= 1
                dst = i + sh if act else None
                if v == nxt:
                    v &= ~1
                reads.append((dst, v))
        for dst, v in reads:
            if dst is not None and dst < L:
                buf[dst] = v
        jg -= 4
    for (k, _), c in zip(surv, cpos):
        if c < L:
            buf[c] = k & ~1 if k == nxt else k
    if nxt == pstar and ppos < WARP * j0:
        buf[ppos] = pstar & ~1
    return buf[:min(psize + S, L)]


def expected(pool, surv, L, nxt):
    allk = sorted(list(pool) + [k for k, _ in surv], key=lambda k: k >> 1)
    return [k & ~1 if k == nxt else k for k in allk[:L]]


def lower_bound(pool, kk):
    lo, hi = 0, len(pool)
    while lo < hi:
        mid = (lo + hi) >> 1
        if (pool[mid] >> 1) < kk:
            lo = mid + 1
        else:
            hi = mid
    return lo


def make_case(rng, L, psize, S, mode):
    ids = rng.sample(range(1, 1 << 20), psize + S)
    dists = sorted(rng.sample(range(1, 1 << 24), psize))
    pool = [(d << 32) | (ids[i] << 1) | rng.randint(0, 1) for i, d in enumerate(dists)]
    last = (pool[-1] >> 1) if psize == L else None
    surv = []
    for t in range(S):
        if mode == "front":
            d = rng.randint(0, dists[0] - 1) if dists and dists[0] > 0 else 0
        elif mode == "tail":
            d = (dists[-1] + rng.randint(1, 1000)) if dists else rng.randint(0, 1000)
        elif mode == "one":
            d = dists[len(dists) // 2] if dists else 5
            d = d + 1 if psize else d
        else:
            d = rng.randint(0, (dists[-1] if dists else 1000) + 50)
        key = (d << 32) | (ids[psize + t] << 1) | 1
        if last is not None and (key >> 1) >= last:
            continue
        surv.append((key, lower_bound(pool, key >> 1)))
    return pool, surv


def test_merge_moves_match_the_merged_pool():
    rng = random.Random(11)
    n = 0
    for trial in range(3000):
        L = rng.choice([10, 31, 32, 33, 64, 100, 128, 200, 400, 448, 512, 1000])
        psize = rng.choice([1, 2, L // 2, L - 1, L, rng.randint(1, L)])
        psize = max(1, min(psize, L))
        S = rng.choice([1, 2, 5, 31, 32, 33, 63, 64])
        mode = rng.choice(["front", "tail", "one", "mixed", "mixed"])
        pool, surv = make_case(rng, L, psize, S, mode)
        if not surv:
            continue
        # the next node: the smaller of the best survivor and the first unvisited entry
        unv = [i for i, k in enumerate(pool) if k & 1]
        ppos = unv[0] if unv else -1
        pstar = pool[ppos] if ppos >= 0 else (1 << 64) - 1
        mk = min(k for k, _ in surv)
        nxt = min(mk, pstar)
        got = kernel_merge(pool, surv, L, nxt, ppos, pstar)
        assert got == expected(pool, surv, L, nxt), (trial, L, psize, len(surv), mode)
        n += 1
    assert n > 2500
