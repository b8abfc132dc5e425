"""Split node records (gann_config.part_count > 1): the records of id range p
live in their own arrays -- on this device (part_index -1) or in another
process's GPU, mapped with gann_part_export / gann_part_attach -- and the
search must return exactly what the single-array layout returns.

The multi-process case runs one child process per GPU (spawned, so no CUDA
state is inherited); each maps the other's range through CUDA IPC and reads it
over NVLink with plain loads. It is skipped on a box with fewer than 2 GPUs.
"""
import multiprocessing as mp
import queue

import numpy as np
import pytest

from conftest import get_index
from gustann_b200.api import (ADC_TABLE, GANN_ESTATE, GANN_OPT_ADC_MODE, GANN_OPT_NEIGHBOUR_CODES, GustANN,
                              GustANNConfig, GustANNError, GustANNStats)
from oracle import F_NAVRACE, Oracle

pytestmark = pytest.mark.gpu


def _cfg(info):
    p = info["paths"]
    return GustANNConfig(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"])


@pytest.mark.parametrize("name", ["u8", "f32", "f32_odd"])
@pytest.mark.parametrize("parts", [2, 3, 8])
def test_split_records_on_one_device_equal_oracle(index_root, name, parts):
    info = get_index(index_root, name)
    whole = GustANN(info["dtype"])
    whole.init_pure_mem(_cfg(info), True)
    split = GustANN(info["dtype"])
    split.init_pure_mem(_cfg(info), True, part_count=parts, part_index=-1)
    p = info["paths"]
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"])
    q = info["queries"]
    try:
        for setup in ("auto", "table", "separate-codes"):
            for g in (whole, split):
                g.set_option(GANN_OPT_ADC_MODE, ADC_TABLE if setup == "table" else 0)
                g.set_option(GANN_OPT_NEIGHBOUR_CODES, 0 if setup == "separate-codes" else 1)
            for ef in (16, 64, 200):
                st = GustANNStats()
                a = whole.query(q, 10, ef)
                b = split.query(q, 10, ef, st)
                for x, y in zip(a, b):
                    np.testing.assert_array_equal(x, y)
                onns, odist, ofound, ohops, oflags = o.search(q, 10, ef)
                ok = (oflags & F_NAVRACE) == 0
                np.testing.assert_array_equal(b[0][ok], onns[ok])
                np.testing.assert_array_equal(b[1][ok], odist[ok])
                assert st.capped_queries == 0
    finally:
        whole.close()
        split.close()
        o.close()


def test_search_needs_every_range(index_root):
    info = get_index(index_root, "f32")
    g = GustANN(info["dtype"])
    g.init_pure_mem(_cfg(info), True, part_count=2, part_index=0)
    try:
        with pytest.raises(GustANNError) as e:
            g.query(info["queries"][:4], 10, 20)
        assert e.value.code == GANN_ESTATE
        blob = g.export_part()
        with pytest.raises(GustANNError):
            g.attach_part(0, blob)          # its own range is already present
        with pytest.raises(GustANNError):
            g.attach_part(1, blob)          # the blob names range 0
    finally:
        g.close()


def _rank_main(rank, world, info, q, ef, blobs_out, blobs_in, results):
    """One process per GPU: load range `rank`, trade blobs, search a query shard."""
    try:
        import torch
        torch.cuda.set_device(rank)
        g = GustANN(info["dtype"], device=rank)
        g.init_pure_mem(_cfg(info), True, part_count=world, part_index=rank)
        for r in range(world):
            if r != rank:
                blobs_out[r].put((rank, g.export_part()))
        for _ in range(world - 1):
            src, blob = blobs_in.get(timeout=120)
            g.attach_part(src, blob)
        shard = np.array_split(np.arange(len(q)), world)[rank]
        nns, dist, found = g.query(q[shard], 10, ef)
        results.put((rank, shard, nns, dist, found, None))
        # keep the exported range mapped until every rank has searched
        blobs_in.get(timeout=120)
        g.close()
    except Exception as e:  # reported to the parent, which fails the test
        results.put((rank, None, None, None, None, repr(e)))


def test_split_records_across_gpus(index_root):
    import torch
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    info = get_index(index_root, "f32")
    p = info["paths"]
    q = info["queries"]
    ef = 64
    ctx = mp.get_context("spawn")
    inboxes = [ctx.Queue() for _ in range(world)]
    results = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, info, q, ef, inboxes, inboxes[r], results))
             for r in range(world)]
    for pr in procs:
        pr.start()
    got = []
    try:
        for _ in range(world):
            got.append(results.get(timeout=600))
    except queue.Empty:
        pass
    finally:
        for ib in inboxes:
            ib.put((-1, b""))               # release the ranks
        for pr in procs:
            pr.join(timeout=120)
            if pr.is_alive():
                pr.kill()
    errors = [g[5] for g in got if g[5]]
    assert len(got) == world and not errors, errors
    o = Oracle(p["index_file"], p["pq_file_prefix"], p["nav_graph_prefix"], info["dtype"])
    onns, odist, ofound, _, oflags = o.search(q, 10, ef)
    o.close()
    for rank, shard, nns, dist, found, _ in got:
        ok = (oflags[shard] & F_NAVRACE) == 0
        np.testing.assert_array_equal(nns[ok], onns[shard][ok])
        np.testing.assert_array_equal(dist[ok], odist[shard][ok])
        np.testing.assert_array_equal(found[ok], ofound[shard][ok])
