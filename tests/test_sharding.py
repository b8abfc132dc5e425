"""Query sharding on CPU ranks (gloo, world_size 2 and 3): every query is
searched exactly once and the gathered result equals the single-process one.
A rank that fails is seen by the others as a collective error, not a hang."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from gustann_b200.sharding import shard_range

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden", "g_u8")


def test_shard_range_partitions():
    for n in (0, 1, 7, 10, 1001):
        for w in (1, 2, 3, 8):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 3, 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, fail_rank):
    import datetime
    import numpy as np
    import torch.distributed as dist
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    from gustann_b200 import formats
    from gustann_b200.sharding import gather_results, search_shard
    from oracle import Oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        p = formats.index_paths(GOLD)
        q = np.load(os.path.join(GOLD, "queries.npy"))
        o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], formats.UINT8)

        def search(qs, k, ef):
            if rank == fail_rank:
                raise RuntimeError("injected rank failure")
            r = o.search(qs, k, ef, threads=1)
            return r[0], r[1], r[2]

        lo, hi, nns, dst, found = search_shard(q, 10, 20, search, rank, world)
        res = gather_results(len(q), 10, lo, nns, dst, found)
        if rank == 0:
            np.savez(os.path.join(out_dir, "res.npz"), nns=res[0], dist=res[1], found=res[2])
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_equals_single(tmp_path, world):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from gustann_b200 import formats
    from oracle import Oracle
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), -1), nprocs=world, start_method="spawn")
    r = np.load(tmp_path / "res.npz")
    p = formats.index_paths(GOLD)
    q = np.load(os.path.join(GOLD, "queries.npy"))
    nns, dist, found, _, _ = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"],
                                    formats.UINT8).search(q, 10, 20)
    assert np.array_equal(r["nns"], nns) and np.array_equal(r["dist"], dist) and np.array_equal(r["found"], found)


def test_failed_rank_is_reported(tmp_path):
    """Rank 1 raises before the gather; rank 0's collective ends with an error
    within the process-group timeout instead of waiting forever."""
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), 1), nprocs=2, start_method="spawn")
    assert (tmp_path / "err1.txt").read_text() == "injected rank failure"
    assert (tmp_path / "err0.txt").exists()
    assert not (tmp_path / "res.npz").exists()


class _FakePartHandle:
    """Stands in for a GustANN handle: records what it exported and attached."""

    def __init__(self, rank):
        self.rank = rank
        self.attached = {}

    def export_part(self):
        return f"range-{self.rank}".encode()

    def attach_part(self, part, blob):
        assert part not in self.attached and part != self.rank
        self.attached[part] = blob


def _exchange_worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    from gustann_b200.sharding import exchange_parts
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        h = _FakePartHandle(rank)
        exchange_parts(h, rank, world)
        with open(os.path.join(out_dir, f"{rank}.txt"), "w") as f:
            f.write(";".join(f"{k}={v.decode()}" for k, v in sorted(h.attached.items())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_parts_gives_every_rank_every_other_range(tmp_path, world):
    mp.spawn(_exchange_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        got = open(tmp_path / f"{r}.txt").read()
        want = ";".join(f"{k}=range-{k}" for k in range(world) if k != r)
        assert got == want
