#!/usr/bin/env python
"""Benchmark: QPS at recall@10 = 0.9 of the in-HBM search path.

One step = one search of the rank's query batch (10k queries, top-10) at the
smallest swept ef_search whose recall@10 against exact ground truth reaches
the target. Workload: configuration 1 (10M x 96-d float32, DEEP-like mixture,
Vamana-style R=64 graph, PQ M=32, pivot graph) on one B200 per rank; ranks
shard the queries (weak scaling, no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0). `value` is device-resident throughput (inputs
in HBM, CUDA events on the launching stream, max over ranks); `e2e` is the
same metric through the C ABI with host buffers (host<->device copies inside
the timed region). The index (6.7 GB) exceeds the 126 MB L2, so no flush is
needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from gustann_b200 import formats  # noqa: E402
from gustann_b200.index import datagen, pipeline  # noqa: E402
from gustann_b200.index.graph import knn_exact  # noqa: E402

METRIC = "QPS at recall@10=0.9 (in-HBM beam search, 1 query batch per step)"
TOPK = 10


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1", choices=list(datagen.CONFIGS))
    ap.add_argument("--points", "--n", dest="n", type=int, default=0,
                    help="override the number of base points (use --points under torchrun: its parser takes --n)")
    ap.add_argument("--nq", type=int, default=10000)
    ap.add_argument("--target", type=float, default=0.9)
    # the sweep stops at the first ef reaching the recall target; steps of 8
    # around the C1 operating point keep that ef close to the smallest that does
    ap.add_argument("--efs", default="32,48,64,80,96,112,128,136,144,152,160,168,176,184,192,200,208,224,240,256,"
                                     "288,320,384,448,512,640,768,1024")
    ap.add_argument("--cache", default=os.environ.get("GANN_BENCH_CACHE", "/tmp/gann_bench"))
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split-records", action="store_true",
                    help="N>1: each rank holds 1/N of the node records and reads the others over NVLink")
    return ap.parse_args()


def spec_for(args) -> datagen.MixtureSpec:
    import dataclasses
    s = datagen.CONFIGS[args.config]
    return dataclasses.replace(s, n=args.n or s.n)


# ------------------------------------------------------------------ plumbing
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            torch.cuda.set_device(self.local)
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(minutes=10),
                                                 device_id=torch.device("cuda", self.local))
            self.pg = True
        elif torch.cuda.is_available():
            torch.cuda.set_device(0)

    def barrier(self):
        if self.pg:
            torch.distributed.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg:
            torch.distributed.destroy_process_group()


class Clocks:
    """nvidia-smi sampling (every 20 ms) around the timed region; stop() keeps
    the samples that arrived inside it (the nearest ones on either side when
    the region is shorter than one period)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        # nvidia-smi numbers GPUs physically; address this process's GPU by UUID
        try:
            self.id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            self.id = str(dev)
        self.p = None
        self.lines = []

    def start(self, wait_s: float = 5.0):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.id}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None
            return
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < wait_s and self.p.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.p.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def stop(self, t_begin: float, t_end: float) -> dict:
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.05)
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        inside = [ln for t, ln in self.lines if t_begin <= t <= t_end + 0.025]
        where = "inside the timed region"
        if not inside:
            before = [ln for t, ln in self.lines if t < t_begin][-1:]
            after = [ln for t, ln in self.lines if t > t_end][:1]
            inside, where = before + after, "nearest samples around a region shorter than the 20 ms period"
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in inside:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window": where}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch(cfg_key: str, n: int, ef: int, hops: int):
    """DRAM bytes (read + write) per launch of the search kernel, from a
    committed ncu summary under profiles/ that names this workload: a line
    `traffic_bytes_per_launch <config> n=<points> ef=<ef> hops=<hops>: <bytes>`.
    The capture at the nearest ef is scaled by expanded nodes (the traffic is
    per hop: one record and one neighbour-code block); the index is rebuilt on
    every machine, so even a capture at the same ef is scaled by this run's
    expanded nodes. Returns (bytes, source) or (None, reason)."""
    d = os.path.join(ROOT, "profiles")
    pat = re.compile(r"^traffic_bytes_per_launch (\S+) n=(\d+) ef=(\d+) hops=(\d+): (\d+)\s*$")
    found = []
    if os.path.isdir(d):
        for name in sorted(os.listdir(d)):
            if not name.endswith(".md"):
                continue
            with open(os.path.join(d, name)) as f:
                for line in f:
                    m = pat.match(line.strip())
                    if m and m.group(1) == cfg_key and int(m.group(2)) == n:
                        found.append((int(m.group(3)), int(m.group(4)), int(m.group(5)), name))
    if found and hops > 0:
        e, h, b, name = min(found, key=lambda t: abs(t[0] - ef))
        return int(b * hops / h), f"ncu capture at ef={e} (profiles/{name}) scaled by expanded nodes {hops}/{h}"
    return None, "no ncu capture of this index committed"


# ------------------------------------------------------------------ data
def ensure_index(spec, args, d: Dist) -> dict:
    key = f"{args.config}_n{spec.n}_R64_M32_v3"
    root = os.path.join(args.cache, key)
    done = os.path.join(root, "DONE")
    paths = formats.index_paths(root)
    if d.rank == 0 and not os.path.exists(done):
        t0 = time.time()
        X = datagen.base_vectors(spec, device="cuda")
        pipeline.build_index(root, X, spec.dtype, R=64, alpha=1.2, M=32, nav_samples=1_000_000)
        del X
        torch.cuda.empty_cache()
        with open(done, "w") as f:
            f.write(f"{time.time() - t0:.1f}\n")
    t0 = time.time()
    while not os.path.exists(done):
        if time.time() - t0 > 3600:
            raise TimeoutError("index build by rank 0 did not finish")
        time.sleep(2)
    return paths


def recall_at(nns: np.ndarray, gt: np.ndarray, k: int = TOPK) -> float:
    """Set-intersection recall@k (bin/utils.hpp:104-116)."""
    hit = 0
    for a, b in zip(nns[:, :k], gt[:, :k]):
        hit += len(set(a.tolist()) & set(b.tolist()))
    return hit / (len(nns) * k)


def ground_truth(spec, Q: np.ndarray) -> np.ndarray:
    X = datagen.base_vectors(spec, device="cuda")
    qt = torch.from_numpy(Q).cuda()
    ids, _ = knn_exact(X, qt, TOPK)
    del X
    torch.cuda.empty_cache()
    return ids.cpu().numpy()


# ------------------------------------------------------------------ arms
def cpu_baseline(paths, dtype, Q, ef, seconds):
    """The oracle (C restatement of the reference path) on the host cores,
    on a bounded sample of the workload's queries."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    orc.build(ref=False)
    o = orc.Oracle(paths["index_file"], paths["pq_file_prefix"], paths["nav_graph_prefix"], dtype)
    cores = os.cpu_count() or 1
    done, t_total, i = 0, 0.0, 0
    batch = max(256, 8 * cores)
    # cycle through the workload's queries until `seconds` of CPU work (at most
    # three passes), so a fast host still gives a stable figure
    while t_total < seconds and done < 3 * len(Q):
        qb = Q[i % len(Q): i % len(Q) + batch]
        t0 = time.perf_counter()
        o.search(qb, TOPK, ef, threads=cores)
        t_total += time.perf_counter() - t0
        done += len(qb)
        i += len(qb)
    o.close()
    return {"value": done / t_total, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{done} query searches over the workload's {len(Q)} queries at ef_search={ef}, "
                      f"{t_total:.1f} s of CPU work"}


def run_reference(args, d: Dist):
    """--impl reference: the reference path's CPU restatement (the reference
    has no CPU search of its own) timed on the host cores; rank 0 only.

    Also reported, as context: the reference's own CUDA kernels (compiled from
    its sources into oracle/_ref) on this GPU, same index, queries and ef --
    given only the queries the oracle shows inside its defined behaviour."""
    if d.rank != 0:
        return
    spec = spec_for(args)
    paths = ensure_index(spec, args, d)
    Q = datagen.as_float_queries(datagen.query_vectors(spec, args.nq, device="cuda", offset=0))
    gt = ground_truth(spec, Q)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    orc.build(ref=False)
    o = orc.Oracle(paths["index_file"], paths["pq_file_prefix"], paths["nav_graph_prefix"], spec.dtype)
    cores = os.cpu_count() or 1
    efs = [int(x) for x in args.efs.split(",")]
    ef, rec, flags = efs[-1], 0.0, None
    for e in efs:
        nns, _, _, _, fl = o.search(Q, TOPK, e, threads=cores)
        rec, flags = recall_at(nns, gt), fl
        if rec >= args.target:
            ef = e
            break
    per_step = min(len(Q), 2000)
    for _ in range(args.warmup):
        o.search(Q[:min(per_step, 256)], TOPK, ef, threads=cores)
    times = []
    for s_ in range(args.steps):
        qb = Q[(s_ * per_step) % len(Q):][:per_step]
        t0 = time.perf_counter()
        o.search(qb, TOPK, ef, threads=cores)
        times.append((time.perf_counter() - t0, len(qb)))
    o.close()
    tot_t = sum(t for t, _ in times)
    tot_q = sum(n for _, n in times)
    v = tot_q / tot_t
    ref_gpu = None
    if orc.RefGPU.available():
        clean = Q[flags == 0]
        r = orc.RefGPU(paths["index_file"], paths["pq_file_prefix"], paths["nav_graph_prefix"], spec.dtype, spec.dim)
        r.search(clean, TOPK, ef)
        rts = [r.search(clean, TOPK, ef)[3] for _ in range(args.steps)]
        r.close()
        ref_gpu = {"value": len(clean) / float(np.mean(rts)), "unit": "queries/s", "ef_search": ef,
                   "queries": int(len(clean)),
                   "what": "the reference's own CUDA kernels (compiled from its sources) on this GPU; "
                           "GustANNStats.run_time: nav + traversal, host translate included"}
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "queries/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_t / len(times),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": config_json(args, spec, ef, rec),
           "cpu_baseline": {"value": v, "unit": "queries/s", "cores": cores, "kind": "port",
                            "sample": f"{per_step} queries per step at ef_search={ef}"},
           "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "reference_gpu": ref_gpu}
    print(json.dumps(out), flush=True)


def config_json(args, spec, ef, rec):
    return {"workload": f"{args.config}: {spec.n} x {spec.dim}-d {'uint8' if spec.dtype == 0 else 'float32'} "
                        f"{spec.kind}-like mixture ({spec.centers} centers), R=64, PQ M=32, pivot graph, "
                        f"{args.nq} queries/rank, top-{TOPK}",
            "ef_search": ef, "recall_at_10": rec, "recall_target": args.target, "queries_per_rank": args.nq,
            "l2_flush": "not needed: index (>6 GB) larger than L2",
            "parallelism": f"query shards x{args.gpus}" + (f", records split x{args.gpus}"
                                                            if getattr(args, "split_records", False) and args.gpus > 1
                                                            else "")}


def run_ours(args, d: Dist):
    from gustann_b200.api import GustANN, GustANNConfig, GustANNStats
    spec = spec_for(args)
    paths = ensure_index(spec, args, d)
    dev = d.local
    Q = datagen.as_float_queries(datagen.query_vectors(spec, args.nq, device="cuda", offset=d.rank))
    gt = ground_truth(spec, Q)
    g = GustANN(spec.dtype, device=dev)
    cfg = GustANNConfig(paths["index_file"], paths["pq_file_prefix"], paths["nav_graph_prefix"])
    split = args.split_records and d.world > 1
    if split:
        from gustann_b200.sharding import exchange_parts
        g.init_pure_mem(cfg, True, part_count=d.world, part_index=d.rank)
        exchange_parts(g, d.rank, d.world)
    else:
        g.init_pure_mem(cfg, True)

    efs = [int(x) for x in args.efs.split(",")]
    sweep = []
    ef, rec = efs[-1], 0.0
    for e in efs:
        nns, _, _ = g.query(Q, TOPK, e)
        r = recall_at(nns, gt)
        sweep.append((e, round(r, 4)))
        if r >= args.target:
            ef, rec = e, r
            break
        rec = r
    # every rank must time the same ef: take the largest chosen one
    ef = int(d.max(float(ef)))
    st = GustANNStats()
    nns, _, _ = g.query(Q, TOPK, ef, st)
    rec = recall_at(nns, gt)
    assert st.capped_queries == 0

    nq = len(Q)
    dq = torch.from_numpy(Q).cuda(dev)
    dn = torch.empty((nq, TOPK), dtype=torch.int32, device=dev)
    dd = torch.empty((nq, TOPK), dtype=torch.float32, device=dev)
    df = torch.empty(nq, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def launch():
        g.search_device(dq.data_ptr(), nq, TOPK, ef, dn.data_ptr(), dd.data_ptr(), df.data_ptr(), 0,
                        stream.cuda_stream)

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize(dev)
    clocks = Clocks(dev)
    clocks.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    d.barrier()
    torch.cuda.synchronize(dev)
    torch.cuda.cudart().cudaProfilerStart()      # a profiler started with --profile-from-start off sees only this
    t_begin = time.perf_counter()
    for a, b in evs:
        a.record(stream)
        launch()
        b.record(stream)
    torch.cuda.synchronize(dev)
    t_end = time.perf_counter()
    torch.cuda.cudart().cudaProfilerStop()
    d.barrier()
    ck = clocks.stop(t_begin, t_end)
    step_ms = [a.elapsed_time(b) for a, b in evs]
    t_step = d.max(float(np.mean(step_ms)))
    total_q = d.sum(float(nq))
    value = total_q / (t_step * 1e-3)

    # e2e: the reference-facing call with host buffers (pinned), copies included
    hq = torch.from_numpy(Q).pin_memory().numpy()
    hn = torch.zeros((nq, TOPK), dtype=torch.int32).pin_memory().numpy()
    hd = torch.zeros((nq, TOPK), dtype=torch.float32).pin_memory().numpy()
    hf = torch.zeros(nq, dtype=torch.int32).pin_memory().numpy()
    for _ in range(args.warmup):
        g.search(hq, nq, TOPK, ef, hn, hd, hf)
    d.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        g.search(hq, nq, TOPK, ef, hn, hd, hf)
    t_e2e = (time.perf_counter() - t0) / args.steps
    d.barrier()
    t_e2e = d.max(t_e2e)
    e2e = {"value": total_q / t_e2e, "unit": "queries/s", "h2d_bytes_per_step": int(Q.nbytes),
           "d2h_bytes_per_step": int(hn.nbytes + hd.nbytes + hf.nbytes)}

    peak, peak_kind = measured_peak()
    achieved = st.bytes_touched / (np.mean(step_ms) * 1e-3) / 1e9
    traffic, traffic_src = traffic_per_launch(args.config, spec.n, ef, int(st.hops))
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
            "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(st.bytes_touched),
            "hops_per_query": st.hops / nq, "adc_per_query": st.adc_evals / nq}

    out = None
    if d.rank == 0:
        cpu = None
        if d.world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(paths, spec.dtype, Q, ef, args.cpu_seconds)
        out = {"metric": METRIC, "value": round(value, 1), "unit": "queries/s", "n_gpus": d.world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_step, 4),
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
               "data": "synthetic", "config": config_json(args, spec, ef, rec), "e2e": e2e,
               "roofline": roof, "cpu_baseline": cpu, "clocks": ck, "gpu_launches": args.steps,
               "recall_sweep": sweep}
    d.barrier()          # split records: peers read this rank's range until every rank is done
    g.close()
    return out


def main():
    args = parse()
    torch.backends.cuda.matmul.allow_tf32 = False
    d = Dist()
    try:
        if args.impl == "reference":
            run_reference(args, d)
        else:
            out = run_ours(args, d)
            if out is not None:
                print(json.dumps(out), flush=True)
    finally:
        d.close()


if __name__ == "__main__":
    main()
