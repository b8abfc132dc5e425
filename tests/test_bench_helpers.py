"""Host-side pieces of bench.py that shape its JSON line: recall@k, the traffic
figure read from the committed ncu summary, and the clock-sample filter."""
import os
import sys

import numpy as np

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_recall_at_counts_set_intersection():
    nns = np.array([[1, 2, 3], [4, 5, 6]])
    gt = np.array([[3, 2, 9], [7, 8, 9]])
    assert bench.recall_at(nns, gt, k=3) == 2 / 6
    assert bench.recall_at(nns, nns, k=3) == 1.0


def test_traffic_scales_the_committed_capture_by_hops():
    b, src = bench.traffic_per_launch("c1", 10_000_000, 176, 0)
    assert b is None
    lines = [ln for ln in open(os.path.join(ROOT, "profiles", "search_kernel_piv_c1_10m_launch_list.md"))
             if ln.startswith("traffic_bytes_per_launch c1 n=10000000")]
    assert len(lines) == 1
    head, val = lines[0].rsplit(":", 1)
    hops = int(head.split("hops=")[1])
    base = int(val)
    b, src = bench.traffic_per_launch("c1", 10_000_000, 176, hops)
    assert b == base and "ef=176" in src
    b2, _ = bench.traffic_per_launch("c1", 10_000_000, 192, 2 * hops)
    assert b2 == 2 * base
    # another point count of the same configuration: the nearest capture, named as such
    b3, src3 = bench.traffic_per_launch("c1", 123, 176, hops)
    assert b3 == base and "10000000-point" in src3
    assert bench.traffic_per_launch("c9", 10_000_000, 176, hops)[0] is None


def test_shards_cover_the_query_set():
    for n in (0, 1, 7, 100_000):
        for world in (1, 2, 3, 8):
            parts = [bench.shard(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))


def test_recall_table_merges_both_arms():
    t = bench.recall_table([(16, 0.5), (24, 0.7)], {"oracle": [[16, 0.5], [24, 0.69]],
                                                   "reference_gpu": [[16, 0.5, 9990]]})
    assert t["rows"][1] == {"ef": 24, "ours": 0.7, "oracle": 0.69, "reference_gpu": None}
    assert abs(t["max_abs_diff_oracle"] - 0.01) < 1e-9 and t["max_abs_diff_reference_gpu"] == 0.0
    assert bench.recall_table([(16, 0.5)], None)["max_abs_diff_oracle"] is None


def test_defaults_name_the_headline_configuration():
    a = bench.parse([])
    assert a.config == "c2" and a.nq == 100_000
    efs = [int(x) for x in a.efs.split(",")]
    assert efs == sorted(efs)
    assert (a.topk, a.pq_chunks, a.metric) == (10, 32, 0)


def test_configuration_4_is_inner_product_top_100():
    a = bench.parse(["--config", "c4"])
    assert (a.topk, a.pq_chunks, a.metric) == (100, 96, 1)
    efs = [int(x) for x in a.efs.split(",")]
    assert efs == sorted(efs) and efs[0] >= a.topk
    c = bench.config_json(a, bench.spec_for(a), efs[0], 0.9, 2)
    assert "recall_at_100" in c and "inner product" in c["workload"] and "Zipf(1.1)" in c["workload"]


def test_clock_samples_inside_the_window():
    c = bench.Clocks.__new__(bench.Clocks)
    c.p = None
    c.lines = []
    assert c.stop(0.0, 1.0)["samples"] == 0                     # no sampler

    class Done:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            return 0

    row = "0, {mhz}, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, {cap}"
    c.p = Done()
    c.lines = [(0.5, row.format(mhz=1000, cap="Not Active")),
               (1.01, row.format(mhz=1965, cap="Active")),
               (1.02, row.format(mhz=1965, cap="Not Active")),
               (3.0, row.format(mhz=900, cap="Not Active"))]
    r = c.stop(1.0, 1.03)
    assert r["samples"] == 2 and r["sm_mhz"] == 1965 and r["reasons"] == ["sw_power_cap"]
    assert r["window"] == "inside the timed region"
    c.lines = [(0.5, row.format(mhz=1500, cap="Not Active")), (3.0, row.format(mhz=1600, cap="Not Active"))]
    r = c.stop(1.0, 1.001)
    assert r["samples"] == 2 and r["window"].startswith("nearest")


def test_sector_rounded_bytes():
    # c2 shape: 128-d uint8, 64 slots, 32 chunks; one query, 2 hops, 100 neighbours
    b = bench.bytes_moved_32(128, 1, 64, 32, 1, 10, 2, 100)
    assert b == 512 + 2 * (128 + 256) + 100 * 32 + 80
    # c1 shape: 96-d float32 (384 B rows), odd sizes round up
    assert bench.bytes_moved_32(96, 4, 61, 30, 1, 1, 1, 1) == 384 + 384 + 256 + 32 + 8
