#!/usr/bin/env python
"""Benchmark of the B200 sampling + aggregation path.

Headline (one JSON line on rank 0): sampled subgraphs/s of the large sharded
workload — 111,059,956 nodes / 1,615,685,872 edges (Zipf(2.0) out-degrees),
bf16 128-d features node-range partitioned across the ranks, 3-hop fanout
[15, 10, 5], 8192 seeds per GPU per step; when N > 1 the feature halo moves
in the bulk peer exchange over NVLink (driver.PeerFeatures). A step = sample
one batch of seeds + gather the features of every sampled node. Synthetic
inputs stand in for the dataset.

At N = 1 the line also carries the standalone CSR SpMM (2,449,029 rows,
61,859,140 nnz, 256 features, fp32 and bf16: achieved HBM GB/s), the temporal
169K-node sampler (fanout [10, 5], 1024 seeds, cutoff = seed timestamp) and
the heterogeneous temporal sampler (4 node sets, 4 edge types, 4096 seeds)
next to their CPU baselines.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dgfx|reference]
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

B_SEEDS = 8192
GRAPH_STEPS = 10  # at most this many large sharded steps per CUDA-graph replay
FANOUT = [15, 10, 5]
FEAT_DIM = 128


def log(*a):
    if int(os.environ.get("RANK", "0")) == 0:
        print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed
    region runs: NVML every millisecond (read-only queries), else nvidia-smi
    every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []  # (sm_mhz, max_mhz, set of active reason names)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = None
            try:  # the torch device's own GPU (NVML ignores CUDA_VISIBLE_DEVICES)
                import torch

                self._h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{torch.cuda.get_device_properties(gpu_index).uuid}")
            except Exception:  # noqa: BLE001
                self._h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self._max = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._bits = {
                "hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap,
            }
        except Exception:  # noqa: BLE001
            self._nvml = None

    def start(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _sample_nvml(self):
        nv = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        self.rows.append((float(sm), float(self._max), {k for k, bit in self._bits.items() if mask & bit}))

    def _sample_smi(self):
        out = subprocess.run(
            ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
            capture_output=True, text=True, timeout=5,
        ).stdout.strip()
        if out:
            r = [x.strip() for x in out.split(",")]
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            if r[1].replace(".", "").isdigit() and r[2].replace(".", "").isdigit():
                self.rows.append((float(r[1]), float(r[2]),
                                  {n for n, v in zip(names, r[5:9]) if v.lower() == "active"}))

    def _run(self):
        while not self._stop.is_set():
            try:
                if self._nvml is not None:
                    self._sample_nvml()
                else:
                    self._sample_smi()
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.001 if self._nvml is not None else 0.2)

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted(set().union(*(r[2] for r in self.rows))), "samples": len(self.rows),
                "source": "nvml" if self._nvml is not None else "nvidia-smi"}


TIMING = {}


def timed(fn, steps, sync_fn, name="timed", finish=None):
    """Device time of `steps` calls bracketed by syncs, inside an NVTX range
    (so profilers can be restricted to the timed region). An event is
    recorded on the launching stream before every call and after the last
    one; the result is the MEDIAN of the per-call intervals in ms (the mean
    over the whole region is kept in TIMING[name]). `finish` joins side
    streams into the timing stream before the end event, so the last
    interval includes their drain."""
    import torch

    sync_fn()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    torch.cuda.nvtx.range_push(name)
    h0 = time.perf_counter()
    for i in range(steps):
        ev[i].record()
        fn(i)
    if finish is not None:
        finish()
    ev[steps].record()
    host_ms = (time.perf_counter() - h0) * 1e3 / steps
    sync_fn()
    torch.cuda.nvtx.range_pop()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total = ev[0].elapsed_time(ev[steps])
    # host_issue_ms: host time per call to enqueue the work; when it is close
    # to mean_ms the GPU waits on the host.
    TIMING[name] = {"median_ms": statistics.median(per), "mean_ms": total / steps, "steps": steps,
                    "min_ms": min(per), "max_ms": max(per), "host_issue_ms": host_ms}
    return statistics.median(per)


def count_dgfx_launches(fn):
    """Kernels of this library launched by one call of fn (CUPTI via the
    torch profiler; names in the dgfx namespace)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    return sum(1 for n in names if "dgfx" in n), len(names)


# ---------------------------------------------------------------------------
# Large sharded sampling (headline).
# ---------------------------------------------------------------------------
def large_spec(scale):
    import dataclasses

    from distributed_graph_flow_b200 import synth

    s = synth.LARGE_SHARDED
    if scale == 1.0:
        return s
    return dataclasses.replace(s, num_nodes=max(1000, int(s.num_nodes * scale)), num_edges=int(s.num_edges * scale))


def setup_large(rank, world, dev, scale=1.0, halo="exchange", cache=0.0, split=True):
    import torch

    from distributed_graph_flow_b200 import driver, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    spec = large_spec(scale)
    t0 = time.time()
    index, _, _ = synth.build_graph(spec, dev)
    t_graph = time.time() - t0
    rpr = math.ceil(spec.num_nodes / world)
    lo = rank * rpr
    cnt = max(0, min(rpr, spec.num_nodes - lo))
    plan = cfg.explicit_plan("paper", "cites", FANOUT)
    cc = ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None],
                                   ext._native.MODE_RANDOM, seed=1234)
    if halo == "nccl":
        table = synth.normal_features(lo, cnt, FEAT_DIM, spec.seed + 100, torch.bfloat16, dev)
        feats = driver.HaloFeatures(table, rpr, rank, world)
    else:
        # Exchange slots sized to the sampler's batch capacity: never overflow.
        slot = B_SEEDS * cc.tree_size if halo == "exchange" else 0
        feats = driver.PeerFeatures(cnt, FEAT_DIM, torch.bfloat16, rpr, spec.num_nodes, rank, world, dev,
                                    exchange_rows=slot)
        synth.normal_features(lo, cnt, FEAT_DIM, spec.seed + 100, torch.bfloat16, dev, out=feats.table)
        feats.connect()
        table = feats.table
        if cache > 0 and world > 1 and halo == "exchange":
            # Read-only copy of the most-referenced rows on every GPU.
            hot = driver.hot_rows(index, int(cache * spec.num_nodes))
            feats.cache_info = {"fraction": cache, "rows": int(hot.numel()),
                                "gb_per_gpu": round(feats.replicate(hot) / 1e9, 2)}
            del hot
    # A second sampler handle (same index, plan and seed) lets overlapped
    # steps alternate workspaces, so one batch's large-tree tail runs beside
    # the next batch's first kernel.
    cc_alt = ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None],
                                       ext._native.MODE_RANDOM, seed=1234) if split else None
    sharded = driver.ShardedSampler(cc, feats, rank, world, cc_alt=cc_alt)
    torch.cuda.synchronize()
    log(f"[bench] large graph built in {t_graph:.1f}s; setup {time.time() - t0:.1f}s; T={cc.tree_size}")
    return spec, index, table, cc, sharded, plan


def bench_large(args, rank, world, dev):
    import torch
    import torch.distributed as dist

    from distributed_graph_flow_b200 import _native, synth

    spec, index, table, cc, sharded, plan = setup_large(rank, world, dev, args.scale, args.halo, args.halo_cache,
                                                        args.split)
    W, K = args.warmup, args.steps
    from distributed_graph_flow_b200 import driver

    # Steps per CUDA-graph replay: the largest divisor of K up to GRAPH_STEPS,
    # so that exactly K steps are timed (a replay ends with its steps drained,
    # so fewer, longer replays overlap more).
    S = max(d for d in range(1, min(K, GRAPH_STEPS) + 1) if K % d == 0)
    use_graph = args.graph and args.overlap and S > 1 and isinstance(sharded.features, driver.PeerFeatures)
    if not use_graph:
        S = 1
    R = K // S
    seeds = synth.uniform_int((W + K) * B_SEEDS, 0, spec.num_nodes, 77 + rank, 5, dev).view(W + K, B_SEEDS)

    def barrier():
        if world > 1:
            dist.barrier()

    def sync():
        torch.cuda.synchronize()
        barrier()

    # Steps are pipelined: the feature gather of step i (second stream)
    # overlaps the sampling of step i + 1; the timed region ends when both
    # streams are done.
    step = sharded.step_overlapped if args.overlap else sharded.step
    for i in range(W):
        step(seeds[i])
    sharded.drain()
    cc.check()
    if use_graph:
        # S pipelined steps per CUDA-graph replay: the host issues one replay
        # (and one seed copy) per S steps instead of ~10 launches per step.
        captured = driver.CapturedSteps(sharded, B_SEEDS, steps=S)
        for _ in range(max(3, -(-W // S))):  # warm-up replays
            captured.replay(seeds[:S])
        torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    if use_graph:
        timed(lambda r: captured.replay(seeds[W + r * S:W + (r + 1) * S]), R, sync, "step")
        ms = TIMING["step"]["mean_ms"] / S  # whole timed region / K
    else:
        ms = timed(lambda i: step(seeds[W + i]), K, sync, "step", finish=sharded.drain)
        if args.overlap:
            # Pipelined steps leave work on side streams, so per-step intervals on
            # the launching stream alternate; the step time is the whole timed
            # region (side streams drained into it) over K.
            ms = TIMING["step"]["mean_ms"]
    clk = clocks.stop()
    cc.check()
    if sharded.cc_alt is not None:
        sharded.cc_alt.check()
    if hasattr(sharded.features, "check"):
        sharded.features.check()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = B_SEEDS * world / (ms_max / 1e3)

    # Per-step sizes (for the byte counts) from one representative step.
    merged, feats, _ = sharded.step(seeds[W])
    torch.cuda.synchronize()
    total_nodes = int(merged.node_offsets[-1].item())
    total_edges = int(merged.edge_offsets[-1].item())
    st = (ctypes_stats(cc))

    # Kernel-level timings on the same inputs (dominant kernels).
    ms_sample = timed(lambda i: cc.sample_merged(seeds[W + i], call_index=10_000 + i, check=False), K, sync,
                      "kernel_sampler")
    st = ctypes_stats(cc)
    ms_gather = None
    from distributed_graph_flow_b200 import driver

    off = merged.node_offsets
    cap = int(merged.node_ids.numel())
    out = torch.empty((cap, FEAT_DIM), dtype=torch.bfloat16, device=dev)
    g = None
    if isinstance(sharded.features, driver.PeerFeatures):
        def g(_):
            sharded.features.gather_range(merged.node_ids, _native.elem_ptr(off, 0), _native.elem_ptr(off, -1), cap,
                                          out)
    elif world == 1:
        def g(_):
            _native.check(_native.lib().dgfx_gather_rows_ranged(
                _native.ptr(table), int(table.shape[0]), FEAT_DIM * 2, _native.ptr(merged.node_ids),
                _native.elem_ptr(off, 0), _native.elem_ptr(off, -1), cap, _native.ptr(out), _native.stream_handle()))
    if g is not None:
        ms_gather = timed(g, K, sync, "kernel_gather")
        del out

    hbm, peak_kind = measured_peaks()
    # Algorithmic bytes per launch.
    sample_bytes = 16 * st[0] + 4 * st[1] + 8 * B_SEEDS + 8 * total_nodes + 16 * total_edges
    gather_bytes = total_nodes * (2 * FEAT_DIM * 2 + 8)
    kernels = {
        "sampler": {"ms": ms_sample, "bytes_per_launch": sample_bytes, "gbs": sample_bytes / ms_sample / 1e6,
                    "rows_expanded": st[0], "neighbours_sampled": st[1]},
    }
    if ms_gather is not None:
        kernels["feature_gather"] = {"ms": ms_gather, "bytes_per_launch": gather_bytes,
                                     "gbs": gather_bytes / ms_gather / 1e6}
    dom = max(kernels, key=lambda k: kernels[k]["ms"])
    traffic = ncu_traffic().get(dom, {}).get("bytes_per_launch")
    roof = {"kernel": dom, "bound": "latency" if dom == "sampler" else "hbm",
            "achieved": round(kernels[dom]["gbs"], 1), "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(kernels[dom]["gbs"] / hbm, 4), "traffic": traffic}
    if dom == "sampler":
        roof["note"] = ("dependent random row / column loads per hop: bound by memory latency, reported against "
                        "the measured HBM copy bandwidth")

    # End to end through the public API with host buffers.
    if args.minimal:
        e2e, launches = None, 0
    else:
        e2e = bench_large_e2e(sharded, seeds, W, K, dev, world, sync)
        launches, _ = count_dgfx_launches(lambda: sharded.step(seeds[W]))
    res = {
        "metric": "sampled subgraphs/sec",
        "value": round(value, 1),
        "unit": "subgraphs/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_max, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int64 ids / bf16 features",
        "data": "synthetic (seeded power-law graph with the sizes of the 1.6B-edge graph; N(0,1) bf16 features)",
        "config": large_config(args, world),
        "workload_stats": {"nodes_per_step_rank0": total_nodes, "edges_per_step_rank0": total_edges,
                           "pipelined": bool(args.overlap),
                           "pipelining": ("the feature gather of step i overlaps the sampling of step i+1 on a "
                                          "second stream" + ("; each sampling call is split over two samplers "
                                                             "(large-tree kernel, scans and compaction of step i "
                                                             "beside the first kernel of step i+1)"
                                                             if args.split else "")) if args.overlap else "none",
                           "step_time": "whole timed region / K" if args.overlap else "median per-step interval",
                           "issue": (f"{S} steps per CUDA-graph replay (one replay and one seed copy per {S} steps)"
                                     if use_graph else "every step's launches issued from the host"),
                           "timing": TIMING.get("step")},
        "clocks": clk,
        "roofline": roof,
        "kernels": kernels,
        "e2e": e2e,
        "gpu_launches": launches * K,
        "gpu_launches_per_step": launches,
    }
    cache_info = getattr(sharded.features, "cache_info", None)
    if cache_info is not None:
        res["workload_stats"]["halo_cache"] = dict(cache_info)
    if world > 1 and isinstance(sharded.features, driver.PeerFeatures):
        res["multi_gpu"] = multi_gpu_checks(args, sharded, spec, seeds, W, K, rank, world, dev, sync)
    return res, (spec, index, table, cc, plan, seeds, W, sharded)


def multi_gpu_checks(args, sharded, spec, seeds, W, K, rank, world, dev, sync):
    """N > 1, outside the timed region (every rank takes the same collective
    steps): (1) the feature rows one step gathered across the ranks equal
    the rows regenerated from the seeded generator, bit for bit, on every
    rank; (2) per-stage times of the bulk exchange (partition, barrier,
    serve, barrier, scatter; medians over K steps, max over ranks); (3) the
    same K steps with the replicated row cache switched off (pure node-range
    partitioning)."""
    import torch
    import torch.distributed as dist

    from distributed_graph_flow_b200 import _native, driver, synth

    feats_obj = sharded.features
    out = {}
    # (1) correctness of the gathered halo rows.
    merged, feats, _ = sharded.step(seeds[W])
    torch.cuda.synchronize()
    n = int(merged.node_offsets[-1].item())
    ids = merged.node_ids[:n]
    exp = synth.normal_rows(ids, FEAT_DIM, spec.seed + 100, torch.bfloat16)
    owner = torch.div(ids, feats_obj.rows_per_rank, rounding_mode="floor")
    remote = owner != rank
    bad = (feats[:n].view(torch.int16) != exp.view(torch.int16)).any(dim=1)
    t = torch.tensor([int(bad.sum().item()), n, int(remote.sum().item())], dtype=torch.int64, device=dev)
    dist.all_reduce(t)
    out["halo_rows_checked"] = int(t[1].item())
    out["halo_rows_remote"] = int(t[2].item())
    out["halo_rows_mismatched"] = int(t[0].item())
    out["halo_rows_bit_exact"] = bool(t[0].item() == 0)
    # (2) per-stage times of the exchange.
    if feats_obj._ex is not None:
        names = ["partition", "barrier_1", "serve", "barrier_2", "scatter"]
        per = {k: [] for k in names}
        cap = int(merged.node_ids.numel())
        buf = torch.empty((cap, feats_obj.dim), dtype=feats_obj.dtype, device=dev)
        for i in range(K):
            m = sharded.cc.sample_merged(seeds[W + i], call_index=20_000 + i * world + rank, check=False)
            ev = []
            feats_obj.gather_range(m.node_ids, _native.elem_ptr(m.node_offsets, 0),
                                   _native.elem_ptr(m.node_offsets, -1), cap, buf, stage_events=ev)
            torch.cuda.synchronize()
            for j, k in enumerate(names):
                per[k].append(ev[j].elapsed_time(ev[j + 1]))
        feats_obj.check()
        med = torch.tensor([statistics.median(per[k]) for k in names], dtype=torch.float64, device=dev)
        dist.all_reduce(med, op=dist.ReduceOp.MAX)
        out["exchange_stage_ms"] = {k: round(float(v), 4) for k, v in zip(names, med.tolist())}
        out["exchange_stage_note"] = "median over steps of each stage alone (not overlapped), max over ranks"
    # (3) the replicated row cache off.
    if feats_obj._replica is not None:
        saved = (feats_obj._replica, feats_obj._hot_slot)
        feats_obj._replica, feats_obj._hot_slot = None, None
        step = sharded.step_overlapped if args.overlap else sharded.step
        for i in range(W):  # as many warm-up steps as the headline (rows of new slots are touched first here)
            step(seeds[i])
        sharded.drain()
        ms = timed(lambda i: step(seeds[W + i]), K, sync, "step_no_cache", finish=sharded.drain)
        if args.overlap:
            ms = TIMING["step_no_cache"]["mean_ms"]  # as the headline: whole timed region / K
        feats_obj.check()
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        feats_obj._replica, feats_obj._hot_slot = saved
        out["no_halo_cache"] = {"value": round(B_SEEDS * world / (float(t.item()) / 1e3), 1), "unit": "subgraphs/s",
                                "ms_per_step": round(float(t.item()), 4),
                                "what": "same steps with the replicated row cache off (pure node-range "
                                        "partitioning: every remote row crosses NVLink)",
                                "timing": TIMING.get("step_no_cache")}
    return out


def large_config(args, world):
    """The headline workload's configuration (identical in both arms)."""
    cfg = {"workload": "large sharded sampling: 111,059,956 nodes, 1,615,685,872 edges, Zipf(2.0), "
                       "fanout [15,10,5], 8192 seeds/GPU, bf16 128-d features node-range partitioned",
           "seeds_per_gpu": B_SEEDS, "fanout": FANOUT, "feature_dim": FEAT_DIM,
           "l2": "inputs larger than L2 (7.4 GB CSR, 28 GB features)",
           "parallelism": f"seed-sharded dp{world}, topology replicated, features node-range partitioned",
           "step": "sample a batch of 8192 seeds + gather every sampled node's features"}
    if args.scale != 1.0:
        cfg["scale"] = args.scale
    if world > 1:
        cfg["halo"] = {"p2p": "peer loads over NVLink (one gather kernel)",
                       "exchange": "bulk peer exchange (bucket by owner, owner-local gather, NVLink pushes, "
                                   "device barrier)",
                       "nccl": "NCCL all-to-all halo exchange"}[args.halo]
        if args.halo == "exchange":
            cfg["halo_cache_fraction"] = args.halo_cache
    return cfg


def ctypes_stats(cc):
    import ctypes

    from distributed_graph_flow_b200 import _native

    out = (ctypes.c_int64 * 3)()
    _native.check(_native.lib().dgfx_sampler_stats(cc._handle, _native.stream_handle(), out))
    return [int(x) for x in out]


def bench_large_e2e(sharded, seeds_dev, W, K, dev, world, sync):
    """Host seeds in, host topology + features out, through the public
    ShardedSampler.step_to_host: seeds copied in, the step sampled and
    gathered, the batch's totals written by the GPU into pinned memory and
    polled, then device-to-host copies of exactly the batch's sizes on a copy
    stream (two sets of pinned host buffers, used in turn, so step i's copies
    run while step i + 1 samples). All copies are inside the timed region."""
    import torch

    from distributed_graph_flow_b200 import driver

    host_seeds = seeds_dev.cpu().pin_memory()
    cap_nodes = B_SEEDS * sharded.cc.tree_size
    hosts = [driver.HostBatch(cap_nodes, FEAT_DIM, torch.bfloat16) for _ in range(2)]
    moved = {"h2d": 0, "d2h": 0}

    def one(i):
        out = sharded.step_to_host(host_seeds[W + i], hosts[i % 2])
        moved["h2d"] += B_SEEDS * 8
        moved["d2h"] += 16 + out.n * 8 + out.m * 16 + (out.n * FEAT_DIM * 2 if sharded.features is not None else 0)

    for i in range(min(W, 2)):
        one(i)
    for h in hosts:
        h.wait()
    moved["h2d"] = moved["d2h"] = 0
    sync()
    t0 = time.perf_counter()
    ms = timed(one, K, sync, "e2e", finish=sharded.drain_host)
    wall = (time.perf_counter() - t0) * 1e3 / K
    t = torch.tensor([max(ms, wall)], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    return {"value": round(B_SEEDS * world / (ms_max / 1e3), 1), "unit": "subgraphs/s",
            "h2d_bytes_per_step": moved["h2d"] // K, "d2h_bytes_per_step": moved["d2h"] // K,
            "ms_per_step": round(ms_max, 3),
            "path": "ShardedSampler.step_to_host: totals published to pinned memory by the GPU and polled; "
                    "copies of step i on a copy stream beside step i + 1"}


# ---------------------------------------------------------------------------
# CPU baseline (oracle / reference code on the host cores).
# ---------------------------------------------------------------------------
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sampler_from_index(index, num_nodes, plan, temporal=False, fill_threads=16):
    from oracle import oracle as O

    rowptr = index.rowptr.cpu().numpy()
    col = index.col.cpu().numpy()
    ts = index.ts.cpu().numpy() if (temporal and index.ts is not None) else None
    ref = O.available(ref=True)
    s = O.OracleSampler.from_csr([num_nodes], [plan.root.nodeset], [plan.root.children[0].edgeset],
                                 {plan.root.children[0].edgeset: (rowptr, col, ts)}, plan, mode=O.MODE_RANDOM,
                                 num_threads=host_cores(), seed=99, temporal=temporal, ref=ref,
                                 fill_threads=fill_threads)
    return s, ("reference" if ref else "port")


def cpu_large_baseline(index, table_host, num_nodes, plan, seeds, budget_s=15.0, threads=None, parity=None):
    """Samples (topology via the reference's compiled samplers when built,
    else the restatement) + numpy feature gather per sample, like
    add_features_to_samples. Returns (subgraphs/s, cores, kind, sample desc,
    parity). With parity = (device FIRST-mode sampler, device seeds), one
    FIRST-mode batch (oldest-first) of the device is first compared with the
    oracle's over the same index, outside the timing."""
    threads = threads or host_cores()
    need = (index.rowptr.numel() + index.col.numel()) * 8 * 1.6 / 1e9 + 4
    if host_mem_gb() < need:
        raise RuntimeError(f"CPU baseline infeasible at this size: needs ~{need:.0f} GB host memory, "
                           f"{host_mem_gb():.0f} GB available")
    s, kind = cpu_sampler_from_index(index, num_nodes, plan)
    par = None
    if parity is not None:
        par = first_mode_parity(s, parity[0], parity[1], None)
    done = 0
    t_sample = t_feat = 0.0
    t_start = time.perf_counter()
    i = 0
    while time.perf_counter() - t_start < budget_s and i < len(seeds):
        batch = seeds[i]
        i += 1
        t0 = time.perf_counter()
        nc, ec, nodes, _, _ = s.sample_raw(batch, threads=threads)
        t1 = time.perf_counter()
        if table_host is not None:
            off = 0
            for c in nc[:, 0]:
                _ = table_host[nodes[off:off + c]]
                off += c
        t_feat += time.perf_counter() - t1
        t_sample += t1 - t0
        done += len(batch)
    rate = done / (t_sample + t_feat)
    return rate, threads, kind, {"seeds": done, "batches": i, "sample_s": round(t_sample, 3),
                                 "feature_gather_s": round(t_feat, 3), "features": table_host is not None}, par


def first_mode_parity(oracle_sampler, device_first, seeds_dev, seed_ts_dev):
    """One FIRST-mode batch (oldest-first under a cutoff; the reference's
    debug_sampling) of the device sampler against the oracle's over the same
    index: True when node ids, local edges and offsets are identical. The
    oracle handle is returned to random mode afterwards."""
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from oracle import oracle as O

    oracle_sampler.set_mode(O.MODE_FIRST)
    try:
        got = ext.batch_to_host(device_first.sample_merged(seeds_dev, seed_ts_dev))
        device_first.check()
        exp = oracle_sampler.sample_merged(seeds_dev.cpu().numpy(),
                                           None if seed_ts_dev is None else seed_ts_dev.cpu().numpy(),
                                           threads=host_cores())
        same = all(np.array_equal(a, b) for a, b in zip(got, exp))
        return {"first_mode_batch_bit_exact": bool(same), "seeds": int(seeds_dev.numel()),
                "nodes": int(got[1][-1]), "edges": int(got[3][-1])}
    finally:
        oracle_sampler.set_mode(O.MODE_RANDOM)


def host_mem_gb():
    try:
        import psutil

        return psutil.virtual_memory().available / 1e9
    except Exception:
        return 0.0


# ---------------------------------------------------------------------------
# Standalone SpMM (products-sized).
# ---------------------------------------------------------------------------
def _scaled(spec, scale):
    import dataclasses

    if scale == 1.0:
        return spec
    return dataclasses.replace(spec, num_nodes=max(1000, int(spec.num_nodes * scale)),
                               num_edges=int(spec.num_edges * scale))


def bench_spmm(dev, steps, scale=1.0):
    import torch

    from distributed_graph_flow_b200 import aggregation, synth

    spec = _scaled(synth.PRODUCTS_SPMM, scale)
    rowptr, _, _ = synth.rowptr_and_edges(spec, dev, with_edges=False)
    nnz = int(rowptr[-1].item())
    col = synth.uniform_int(nnz, 0, spec.num_nodes, 3, 7, dev).to(torch.int32)
    deg = (rowptr[1:] - rowptr[:-1]).clamp_min(1).to(torch.float32)
    row_of = torch.repeat_interleave(torch.arange(spec.num_nodes, device=dev), rowptr[1:] - rowptr[:-1])
    val = (1.0 / deg)[row_of].contiguous()
    del row_of
    F = 256
    hbm, peak_kind = measured_peaks()
    out = {"workload": "CSR SpMM 2,449,029 x 2,449,029, 61,859,140 nnz (Zipf 1.9 rows, max 17,000), x256, "
                       "vals = 1/row_degree", "nnz": nnz}
    ws = aggregation.spmm_workspace(spec.num_nodes, nnz, F, dev)
    for dt, name in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        x = synth.normal_features(0, spec.num_nodes, F, 5, dt, dev)
        y = torch.empty_like(x)
        for _ in range(3):
            aggregation.csr_spmm(rowptr, col, x, val=val, out=y, workspace=ws)
        ms = timed(lambda i: aggregation.csr_spmm(rowptr, col, x, val=val, out=y, workspace=ws), steps,
                   torch.cuda.synchronize, f"spmm_{name}")
        e = x.element_size()
        alg = 8 * (spec.num_nodes + 1) + nnz * 8 + nnz * F * e + spec.num_nodes * F * e
        gbs = alg / ms / 1e6
        out[name] = {"ms": round(ms, 3), "algorithmic_bytes": alg, "achieved_gbs": round(gbs, 1), "peak_gbs": hbm,
                     "peak_kind": peak_kind, "frac": round(gbs / hbm, 4),
                     "traffic": ncu_traffic().get(f"spmm_{name}", {}).get("bytes_per_launch")}
        del x, y
    # CPU baseline: torch-CPU sparse CSR @ dense (fp32) on all host cores
    # over a bounded row sample (jax is not installed, so jax.ops.segment_sum
    # on CPU cannot run; torch's CSR SpMM stands in for it).
    try:
        th = host_cores()
        torch.set_num_threads(th)
        rows = 400_000
        rp = rowptr[: rows + 1].cpu()
        nnz_s = int(rp[-1])
        c = col[:nnz_s].cpu().long()
        v = val[:nnz_s].cpu()
        xh = synth.normal_features(0, spec.num_nodes, F, 5, torch.float32, dev).cpu()
        a = torch.sparse_csr_tensor(rp, c, v, size=(rows, spec.num_nodes))
        _ = torch.sparse.mm(a, xh)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 8.0:
            _ = torch.sparse.mm(a, xh)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        alg = 8 * (rows + 1) + nnz_s * 8 + nnz_s * F * 4 + rows * F * 4
        out["cpu_baseline"] = {"value": round(alg / dt / 1e9, 2), "unit": "GB/s (same byte count)", "cores": th,
                               "kind": "port (torch-CPU CSR SpMM stands in for jax.ops.segment_sum on CPU)",
                               "sample": f"first {rows} rows ({nnz_s} nnz), fp32, {reps} reps, "
                                         f"{dt * 1e3:.1f} ms each"}
        out["speedup_vs_cpu_fp32"] = round(out["fp32"]["achieved_gbs"] / out["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        out["cpu_baseline"] = {"unavailable": str(exc)}
    return out


# ---------------------------------------------------------------------------
# Temporal 169K-node sampler.
# ---------------------------------------------------------------------------
def bench_temporal(dev, steps, scale=1.0, streams=8):
    """Temporal 169K-node sampler, batches of 1024 seeds, each step = sample
    (cutoff = seed timestamp) + gather the fp32 features of the sampled
    nodes + mean aggregation over the sampled subgraph (every node's mean of
    the features of the neighbours it sampled; jax.ops.segment_sum mean
    pooling of hetero_gnn.py:282-294). Reported: one batch per step on one
    stream (eager launches, and one CUDA graph per batch: the per-batch
    latency a training loop sees, the headline here) and `streams`
    independent batches forked inside one graph (throughput)."""
    import torch

    from distributed_graph_flow_b200 import _native, aggregation, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    spec = _scaled(synth.TEMPORAL_169K, scale)
    index, ts, _ = synth.build_graph(spec, dev)
    node_ts = synth.uniform_int(spec.num_nodes, 0, 50, spec.seed, 12, dev)
    table = synth.normal_features(0, spec.num_nodes, FEAT_DIM, 9, torch.float32, dev)
    plan = cfg.explicit_plan("v", "e", [10, 5])
    cc = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], _native.MODE_RANDOM,
                                   seed=3, has_temporal=True)
    B = 1024
    steps = max(steps, 200)  # batches are ~10 us: time enough of them
    nb = 8 + steps
    seeds = synth.uniform_int(nb * B, 0, spec.num_nodes, 21, 9, dev).view(nb, B)
    sts = node_ts[seeds]
    cap = B * cc.tree_size
    feats = torch.empty((cap, FEAT_DIM), dtype=torch.float32, device=dev)
    aggs = torch.empty((cap, FEAT_DIM), dtype=torch.float32, device=dev)

    def step(i):
        m = cc.sample_merged(seeds[i], sts[i], None, call_index=i, check=False)
        off = m.node_offsets
        _native.check(_native.lib().dgfx_gather_rows_ranged(
            _native.ptr(table), spec.num_nodes, FEAT_DIM * 4, _native.ptr(m.node_ids), _native.elem_ptr(off, 0),
            _native.elem_ptr(off, -1), int(m.node_ids.numel()), _native.ptr(feats), _native.stream_handle()))
        aggregation.batch_mean_aggregate(m, feats, out=aggs)
        return m

    for i in range(5):
        step(i)
    cc.check()
    ms_eager = timed(lambda i: step(8 + i), steps, torch.cuda.synchronize, "temporal_eager")
    cc.check()
    samplers = [ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None],
                                          _native.MODE_RANDOM, seed=3 + k, has_temporal=True)
                for k in range(streams)]
    # One batch at a time on one stream: `streams` consecutive batches per
    # graph replay, so the host's launch cost per replay is amortised and the
    # time is the device's per-batch latency.
    single = ext.CapturedSampleStep(samplers[0], B, True, table, aggregate=True)
    for i in range(4):
        single.run(seeds[i], sts[i])
    ms_single = timed(lambda i: single.run(seeds[8 + i], sts[8 + i]), steps, torch.cuda.synchronize,
                      "temporal_single_replay", finish=single.wait)
    del single
    one = ext.CapturedSampleStep(samplers, B, True, table, aggregate=True, serial=True)
    reps_s = max(3, steps // streams)
    for i in range(3):
        one.run(seeds[i * streams:(i + 1) * streams], sts[i * streams:(i + 1) * streams])
    ms_graph = timed(lambda i: one.run(seeds[8 + i * streams:8 + (i + 1) * streams],
                                       sts[8 + i * streams:8 + (i + 1) * streams]),
                     reps_s, torch.cuda.synchronize, "temporal_graph", finish=one.wait) / streams
    del one
    multi = ext.CapturedSampleStep(samplers, B, True, table, aggregate=True)
    reps = steps // streams
    for i in range(4):
        multi.run(seeds[i * streams:(i + 1) * streams], sts[i * streams:(i + 1) * streams])
    ms_multi = timed(lambda i: multi.run(seeds[8 + i * streams:8 + (i + 1) * streams],
                                         sts[8 + i * streams:8 + (i + 1) * streams]),
                     reps, torch.cuda.synchronize, "temporal", finish=multi.wait) / streams
    for smp in samplers:
        smp.check()
    del multi
    out = {"workload": "temporal 169,343 nodes / 1,166,243 edges, Zipf(2.1), ts in [0,50), fanout [10,5], "
                       "1024 seeds per batch, cutoff = seed ts, fp32 128-d features, then mean aggregation over the "
                       "sampled subgraph",
           "step": "sample + feature gather + mean aggregation over the sampled subgraph (one kernel), one batch",
           "value": round(B / (ms_graph / 1e3), 1), "unit": "subgraphs/s", "ms_per_batch": round(ms_graph, 4),
           "mode": f"one batch of 1024 seeds at a time on one stream ({streams} consecutive batches per "
                   f"CUDA-graph replay, time per batch)",
           "eager": {"value": round(B / (ms_eager / 1e3), 1), "ms_per_batch": round(ms_eager, 4)},
           "one_batch_per_replay": {"value": round(B / (ms_single / 1e3), 1), "ms_per_batch": round(ms_single, 4),
                                    "note": "one graph replay per batch issued from Python (one native call: "
                                            "input copies + graph launch on the caller's stream)"},
           f"{streams}_batches_per_replay": {"value": round(B / (ms_multi / 1e3), 1),
                                             "ms_per_batch": round(ms_multi, 4),
                                             "mode": f"{streams} independent batches forked onto {streams} streams "
                                                     "inside one CUDA graph"}}
    # CPU baseline on the same graph and seeds (+ the FIRST-mode parity batch).
    try:
        from oracle import oracle as O

        s, kind = cpu_sampler_from_index(index, spec.num_nodes, plan, temporal=True)
        first = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], _native.MODE_FIRST,
                                          seed=3, has_temporal=True)
        par = first_mode_parity(s, first, seeds[0], sts[0])
        # The aggregation of that batch against the float64 restatement.
        m = first.sample_merged(seeds[0], sts[0])
        f0 = aggregation.gather_rows(table, m.node_ids)
        a0 = aggregation.batch_mean_aggregate(m, f0)
        nodes_h, off_h, edges_h, eoff_h = ext.batch_to_host(m)
        n0 = int(off_h[-1])
        fh = table.cpu().numpy()[nodes_h]
        exp = O.batch_mean_aggregate(off_h, eoff_h, edges_h, fh)
        mag = O.batch_mean_aggregate(off_h, eoff_h, edges_h, np.abs(fh))
        err = np.abs(a0[:n0].cpu().numpy() - exp)
        par["mean_aggregation_within_1e-5"] = bool(np.all(err <= 1e-5 * np.maximum(mag, 1e-30) + 1e-30))
        del first
        th = host_cores()
        host_tab = table.cpu().numpy()
        seeds_h = seeds.cpu().numpy()
        sts_h = sts.cpu().numpy()
        done, t_tot, t_agg = 0, 0.0, 0.0
        i = 0
        while t_tot < 10.0 and i < nb:
            t0 = time.perf_counter()
            nc, ec, nodes, esrc, edst = s.sample_raw(seeds_h[i], sts_h[i], threads=th)
            rows, off = [], 0
            for c in nc[:, 0]:  # add_features_to_samples: one gather per sample
                rows.append(host_tab[nodes[off:off + c]])
                off += c
            t1 = time.perf_counter()
            cpu_mean_aggregate(nc[:, 0], ec[:, 0], esrc, edst, np.concatenate(rows))
            t2 = time.perf_counter()
            t_tot += t2 - t0
            t_agg += t2 - t1
            done += B
            i += 1
            if i == nb:
                i = 0
        out["cpu_baseline"] = {"value": round(done / t_tot, 1), "unit": "subgraphs/s", "cores": th, "kind": kind,
                               "sample": f"{done} seeds: topology ({kind} sampler, {th} threads) + numpy feature "
                                         f"gather per sample + numpy mean aggregation over the merged batch "
                                         f"({t_agg:.2f} s of {t_tot:.2f} s)"}
        out["speedup_vs_cpu"] = round(out["value"] / out["cpu_baseline"]["value"], 1)
        out["parity"] = par
    except Exception as exc:  # noqa: BLE001
        out["cpu_baseline"] = {"unavailable": str(exc)}
    return out


def cpu_mean_aggregate(node_counts, edge_counts, esrc, edst, feats):
    """Mean of the sampled neighbours' features for every node of a merged
    batch on the host (numpy; sources are sorted within a sample, so batch
    sources are sorted and np.add.reduceat sums each node's run)."""
    n_off = np.concatenate([[0], np.cumsum(node_counts)])
    samp = np.repeat(np.arange(len(edge_counts)), edge_counts)
    gsrc = n_off[:-1][samp] + esrc
    gdst = n_off[:-1][samp] + edst
    out = np.zeros_like(feats)
    if len(gsrc):
        starts = np.flatnonzero(np.concatenate([[True], gsrc[1:] != gsrc[:-1]]))
        sums = np.add.reduceat(feats[gdst], starts, axis=0)
        cnt = np.diff(np.concatenate([starts, [len(gsrc)]]))
        out[gsrc[starts]] = sums / cnt[:, None]
    return out


def bench_sage(dev, steps, scale=1.0):
    """GraphSAGE-mean layer forward: mean SpMM over in-neighbours (bf16 out)
    then relu(concat[x, agg] @ W^T + b) on the tensor cores. 2,000,000 nodes,
    40,000,000 edges (Zipf 2.1 generator), bf16 x [N, 256], W [256, 512]
    Glorot-uniform (seeded)."""
    import torch

    from distributed_graph_flow_b200 import aggregation, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    N = max(1024, int(2_000_000 * scale))
    E = max(1024, int(40_000_000 * scale))
    F, F_OUT = 256, 256
    spec = synth.GraphSpec(N, E, 2.1, 20_000, seed=5)
    _, src, dst = synth.rowptr_and_edges(spec, dev)
    idx = ext.build_adjacency_index_device(src, dst, None, N, N, True, False)  # rows = targets
    del src, dst
    x = synth.normal_features(0, N, F, 6, torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(11)
    lim = (6.0 / (2 * F + F_OUT)) ** 0.5
    w = ((torch.rand((F_OUT, 2 * F), generator=g, device=dev) * 2 - 1) * lim).to(torch.bfloat16)
    b = torch.zeros(F_OUT, dtype=torch.float32, device=dev)
    agg = torch.empty((N, F), dtype=torch.bfloat16, device=dev)
    y = torch.empty((N, F_OUT), dtype=torch.bfloat16, device=dev)
    ws = aggregation.spmm_workspace(N, E, F, dev)
    rowptr, col = idx.rowptr, idx.col

    def layer(_):
        aggregation.sage_mean_linear_relu(rowptr, col, x, w, b, agg=agg, workspace=ws, out=y)

    def spmm(_):
        aggregation.csr_spmm(rowptr, col, x, normalize=True, out=agg, workspace=ws)

    def dense(_):
        aggregation.dense_concat(x, agg, w, b, relu=True, out=y)

    for _ in range(3):
        layer(0)
    aggregation.dense_check()
    ms_layer = timed(layer, steps, torch.cuda.synchronize, "sage_layer")
    ms_spmm = timed(spmm, steps, torch.cuda.synchronize, "sage_spmm")
    ms_dense = timed(dense, steps, torch.cuda.synchronize, "sage_dense")
    aggregation.dense_check()
    hbm, kind = measured_peaks()
    tflops_peak = measured_tflops()
    spmm_bytes = 8 * (N + 1) + 4 * E + 2 * F * E + 2 * F * N
    dense_flops = 2.0 * N * (2 * F) * F_OUT
    dense_bytes = 2 * N * (2 * F) + 2 * N * F_OUT + 2 * F_OUT * 2 * F
    out = {"workload": "GraphSAGE-mean forward: 2,000,000 nodes, 40,000,000 edges (Zipf 2.1), bf16 x [N,256], "
                       "mean SpMM -> concat[x, agg] [N,512] -> Dense 512->256 (tcgen05, fp32 accum) + ReLU",
           "value": round(N / (ms_layer / 1e3), 1), "unit": "nodes/s", "ms_per_layer": round(ms_layer, 4),
           "spmm": {"ms": round(ms_spmm, 4), "bytes": spmm_bytes, "gbs": round(spmm_bytes / ms_spmm / 1e6, 1),
                    "frac_hbm": round(spmm_bytes / ms_spmm / 1e6 / hbm, 4), "bound": "hbm"},
           "dense": {"ms": round(ms_dense, 4), "tflops": round(dense_flops / ms_dense / 1e9, 1),
                     "frac_tensor": round(dense_flops / ms_dense / 1e9 / tflops_peak, 4),
                     "gbs": round(dense_bytes / ms_dense / 1e6, 1),
                     "frac_hbm": round(dense_bytes / ms_dense / 1e6 / hbm, 4),
                     "bound": "hbm (AI = 2*512*256/(2*(512+256)) = 170 flop/B, below the ridge)"},
           "peaks": {"hbm_gbs": hbm, "bf16_tflops": tflops_peak, "kind": kind}}
    # CPU baseline: the same layer in torch fp32 on the host cores, on a
    # bounded sample of target rows (their in-edges and rows of x).
    try:
        th = host_cores()
        torch.set_num_threads(th)
        rows = min(N, 50_000)
        rp = rowptr[: rows + 1].cpu()
        c = col[: int(rp[-1])].cpu().long()
        xh = x.float().cpu()
        wh = w.float().cpu()
        bh = b.cpu()
        seg = torch.repeat_interleave(torch.arange(rows), torch.diff(rp))
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 10.0:
            aggh = torch.zeros((rows, F)).index_add_(0, seg, xh[c])
            aggh /= torch.diff(rp).clamp(min=1).float()[:, None]
            _ = torch.relu(torch.cat([xh[:rows], aggh], 1) @ wh.t() + bh)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        out["cpu_baseline"] = {"value": round(rows / dt, 1), "unit": "nodes/s", "cores": th, "kind": "port",
                               "sample": f"{rows} target rows ({int(rp[-1])} in-edges), torch fp32 index_add_ "
                                         f"mean + matmul + relu, {reps} reps"}
        out["speedup_vs_cpu"] = round(out["value"] / out["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        out["cpu_baseline"] = {"unavailable": str(exc)}
    return out


def bench_gat(dev, steps, scale=1.0):
    """Graph-attention aggregation (segment softmax + weighted segment sum):
    2,000,000 target nodes, 40,000,000 edges grouped by target (in-degrees
    from the Zipf 2.1 generator's popularity), 8 heads x 32 dims, bf16
    messages, fp32 logits, bf16 output."""
    import torch

    from distributed_graph_flow_b200 import aggregation, synth

    N = max(1024, int(2_000_000 * scale))
    E = max(1024, int(40_000_000 * scale))
    H, D = 8, 32
    spec = synth.GraphSpec(N, E, 2.1, 20_000, seed=8)
    _, _, dst = synth.rowptr_and_edges(spec, dev)
    ids = torch.sort(dst).values
    del dst
    g = torch.Generator(device=dev).manual_seed(5)
    logits = torch.randn((E, H), generator=g, device=dev)
    msgs = synth.normal_features(0, E, H * D, 12, torch.bfloat16, dev).view(E, H, D)
    out = torch.empty((N, H, D), dtype=torch.bfloat16, device=dev)

    def run(_):
        aggregation.segment_softmax(logits, msgs, ids, N, indices_are_sorted=True)

    for _ in range(3):
        run(0)
    ms = timed(run, max(5, steps // 2), torch.cuda.synchronize, "gat")
    hbm, kind = measured_peaks()
    nbytes = E * (H * D * 2 + H * 4 + 8) + N * H * D * 2 + 8 * (N + 1)
    res = {"workload": "segment softmax + weighted segment sum (GAT relation attention): 2,000,000 targets, "
                       "40,000,000 edges grouped by target, 8 heads x 32, bf16 messages, fp32 logits",
           "ms": round(ms, 4), "algorithmic_bytes": nbytes, "achieved_gbs": round(nbytes / ms / 1e6, 1),
           "peak_gbs": hbm, "peak_kind": kind, "frac": round(nbytes / ms / 1e6 / hbm, 4), "bound": "hbm"}
    del out
    try:  # torch-CPU fp32 on a bounded prefix of the segments
        th = host_cores()
        torch.set_num_threads(th)
        rows = min(N, 100_000)
        n_items = int(torch.searchsorted(ids, torch.tensor(rows, device=dev)).item())
        li, mi, ti = logits[:n_items].cpu(), msgs[:n_items].float().cpu(), ids[:n_items].cpu()
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 8.0:
            mx = torch.full((rows, H), -float("inf")).scatter_reduce(0, ti[:, None].expand(-1, H), li, reduce="amax")
            ex = torch.exp(li - mx[ti])
            den = torch.zeros((rows, H)).index_add_(0, ti, ex)
            w = ex / (den[ti] + 1e-9)
            _ = torch.zeros((rows, H, D)).index_add_(0, ti, w[..., None] * mi)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        cpu_gbs = (n_items * (H * D * 4 + H * 4 + 8) + rows * H * D * 4) / dt / 1e9
        res["cpu_baseline"] = {"value": round(n_items / dt, 1), "unit": "edges/s", "cores": th, "kind": "port",
                               "sample": f"{rows} segments ({n_items} edges), torch fp32 scatter_reduce/index_add_, "
                                         f"{reps} reps ({cpu_gbs:.1f} GB/s)"}
        res["edges_per_s"] = round(E / (ms / 1e3), 1)
        res["speedup_vs_cpu"] = round(res["edges_per_s"] / res["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        res["cpu_baseline"] = {"unavailable": str(exc)}
    return res


def bench_rw_negatives(dev, steps, scale=1.0):
    """Random-walk negative sampling for link prediction on the 169,343-node
    Zipf(2.1) graph (no timestamps: walks ignore them): plan fanout [10, 5]
    (two hops), 5 negatives per seed, 10 walks per negative (the link
    generator's default: 50 walks), 16,384 seeds per call."""
    import dataclasses

    import torch

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    spec = dataclasses.replace(_scaled(synth.TEMPORAL_169K, scale), ts_range=None)
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("v", "e", [10, 5])
    cc = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], _native.MODE_RANDOM, seed=5)
    B, K, W = 16384, 5, 50
    nb = 4 + steps
    seeds = synth.uniform_int(nb * B, 0, spec.num_nodes, 23, 9, dev).view(nb, B)

    def step(i):
        cc.random_walk_negatives(seeds[i], 0, W, K, call_index=i, check=False)

    for i in range(3):
        step(i)
    cc.check_random_walk_negatives()
    ms = timed(lambda i: step(4 + i), steps, torch.cuda.synchronize, "rw_negatives")
    cc.check_random_walk_negatives()
    steps_per_walk = 2
    res = {"workload": "random-walk negatives: 169,343 nodes / 1,166,243 edges Zipf(2.1), plan fanout [10,5], "
                       "5 negatives x 10 walks per seed, 16,384 seeds per call",
           "value": round(B / (ms / 1e3), 1), "unit": "seeds/s", "ms_per_call": round(ms, 4),
           "walk_steps_per_s": round(B * W * steps_per_walk / (ms / 1e3), 1), "bound": "latency (dependent "
           "random row loads per walk step)"}
    try:
        from oracle import oracle as O

        s, kind = cpu_sampler_from_index(index, spec.num_nodes, plan)
        th = host_cores()
        seeds_h = seeds.cpu().numpy()
        done, t_tot, i = 0, 0.0, 0
        while t_tot < 10.0 and i < nb:
            t0 = time.perf_counter()
            s.random_walk_negatives(seeds_h[i], 0, W, K, kind=0, threads=th)
            t_tot += time.perf_counter() - t0
            done += B
            i += 1
        res["cpu_baseline"] = {"value": round(done / t_tot, 1), "unit": "seeds/s", "cores": th, "kind": "port",
                               "sample": f"{done} seeds; restated RandomWalkNegativeSamplerHelper (std::mt19937_64)"
                                         + (" over the reference's compiled AdjacencyIndex" if kind == "reference"
                                            else "")}
        res["speedup_vs_cpu"] = round(res["value"] / res["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        res["cpu_baseline"] = {"unavailable": str(exc)}
    return res


def bench_id_map(dev, steps, scale=1.0):
    """GF graph loading's raw-id join on the device: a 2,449,029-node set with
    12-byte ids ("p" + 11 digits, shuffled) indexed, then both endpoints of
    61,859,140 edges (the products-sized generator) looked up, ids resident in
    HBM. One step = index build + 2 x 61.9M lookups."""
    import torch

    from distributed_graph_flow_b200 import synth
    from distributed_graph_flow_b200.io import ids as ids_lib

    spec = _scaled(synth.PRODUCTS_SPMM, scale)
    N = spec.num_nodes
    _, src, dst = synth.rowptr_and_edges(spec, dev)
    E = int(src.numel())
    g = torch.Generator(device=dev).manual_seed(11)
    perm = torch.randperm(N, generator=g, device=dev)
    W = 12
    node_ids = torch.empty((N, W), dtype=torch.uint8, device=dev)
    node_ids[:, 0] = ord("p")
    v = perm.clone()
    for d in range(W - 1, 0, -1):
        node_ids[:, d] = (v % 10 + 48).to(torch.uint8)
        v //= 10
    del v, perm
    q_src = node_ids[src]
    q_dst = node_ids[dst]
    del src, dst
    torch.cuda.synchronize()
    out = torch.empty((2, E), dtype=torch.int64, device=dev)

    def step(_):
        ix = ids_lib.IdIndex(node_ids, dev)
        ix.lookup(q_src, out=out[0])
        ix.lookup(q_dst, out=out[1])

    for i in range(3):
        step(i)
    ms = timed(step, max(3, steps // 4), torch.cuda.synchronize, "id_map")
    ix = ids_lib.IdIndex(node_ids, dev)
    ms_lookup = timed(lambda _: ix.lookup(q_src, out=out[0]), max(3, steps // 4), torch.cuda.synchronize,
                      "id_lookup")
    hbm, kind = measured_peaks()
    # Per lookup: the 12-byte query, one 8-byte table word, the 12 matched
    # id bytes, the 8-byte result.
    nbytes = E * (W + 8 + W + 8)
    res = {"workload": "raw-id join of GF loading: 2,449,029 node ids (12 bytes) indexed, 2 x 61,859,140 edge "
                       "endpoints looked up; ids in HBM", "value": round(2 * E / (ms / 1e3), 1), "unit": "ids/s",
           "ms_per_step": round(ms, 3), "lookup_ms_per_61.9M": round(ms_lookup, 3),
           "lookup_achieved_gbs": round(nbytes / ms_lookup / 1e6, 1), "peak_gbs": hbm, "peak_kind": kind,
           "lookup_frac": round(nbytes / ms_lookup / 1e6 / hbm, 4), "bound": "hbm (random 32-byte sectors)"}
    try:
        from oracle import oracle as O

        th = host_cores()
        idx_h = node_ids.cpu().numpy().reshape(-1).view(f"S{W}")
        q_h = q_src[:6_000_000].cpu().numpy().reshape(-1).view(f"S{W}")
        empty = q_h[:0]

        def best(fn, reps=2):
            t = []
            for _ in range(reps):
                t0 = time.perf_counter()
                fn()
                t.append(time.perf_counter() - t0)
            return min(t)

        build = best(lambda: O.bytes_map(idx_h, empty, threads=th))
        with_q = best(lambda: O.bytes_map(idx_h, q_h, threads=th))
        lookup_s = max(with_q - build, 1e-3 * with_q)
        rate = len(q_h) / lookup_s
        whole = build + 2 * E / rate
        res["cpu_baseline"] = {"value": round(2 * E / whole, 1), "unit": "ids/s", "cores": th, "kind": "port",
                               "sample": f"restated ByteIdToIdxMapper (std::unordered_map over string views, "
                                         f"{th} threads): index build {build:.2f} s (timed alone) + "
                                         f"{rate / 1e6:.1f} M lookups/s (6M queries), best of 2 each, "
                                         f"extrapolated to 2 x {E} lookups"}
        res["speedup_vs_cpu"] = round(res["value"] / res["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        res["cpu_baseline"] = {"unavailable": str(exc)}
    return res


def measured_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        for k in ("bf16_tflops", "bf16_tflops_burst"):
            if k in d:
                return float(d[k])
    return 1590.0


def bench_hetero(dev, steps, scale=1.0):
    """Heterogeneous temporal sampling: 4 node sets / 4 edge types, edge
    times propagated from node set A's creation years, A seeds with cutoff =
    seed year, both directions of every edge type, per-hop widths [15, 10];
    fp32 128-d features of every sampled A node gathered."""
    import torch

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    spec = synth.scaled_hetero(synth.HETERO_TEMPORAL, scale)
    t0 = time.time()
    g = synth.build_hetero_graph(spec, dev)
    t_build = time.time() - t0
    plan = synth.hetero_plan(spec, "A", [15, 10])
    cc = ext.create_device_sampler(plan, g.nodeset_names, g.num_nodes, g.edgeset_names, g.fwd, g.bwd,
                                   _native.MODE_RANDOM, seed=3, has_temporal=True)
    a = g.nodeset_names.index("A")
    n_a = g.num_nodes[a]
    table = g.features["A"]
    B = 4096
    nb = 8 + steps
    seeds = synth.uniform_int(nb * B, 0, n_a, 23, 9, dev).view(nb, B)
    sts = g.node_ts["A"][seeds]
    feats = torch.empty((B * cc.tree_size, FEAT_DIM), dtype=torch.float32, device=dev)

    def step(i):
        m = cc.sample_merged(seeds[i], sts[i], None, call_index=i, check=False)
        off = m.node_offsets  # node set A's rows: [off[a * B], off[(a + 1) * B])
        _native.check(_native.lib().dgfx_gather_rows_ranged(
            _native.ptr(table), n_a, FEAT_DIM * 4, _native.ptr(m.node_ids), _native.elem_ptr(off, a * B),
            _native.elem_ptr(off, (a + 1) * B), int(m.node_ids.numel()), _native.ptr(feats),
            _native.stream_handle()))

    for i in range(5):
        step(i)
    cc.check()
    ms_serial = timed(lambda i: step(8 + i), steps, torch.cuda.synchronize, "hetero")
    cc.check()
    m = cc.sample_merged(seeds[8], sts[8], None, call_index=8, check=False)
    nodes = int(m.node_offsets[-1].item())

    # Pipelined as the headline step: two samplers over the same index and
    # seed alternate, each call split (warp kernel on the main stream; the
    # large-tree and padded kernels, scans and compaction on the sampler's
    # tail stream), and the A-feature gather on a high-priority stream, so
    # call i's tail and gather overlap call i + 1's. S such steps are captured
    # in one CUDA graph (random streams from the samplers' device counters),
    # so the host issues one replay per S steps, as for the headline.
    cc_alt = ext.create_device_sampler(plan, g.nodeset_names, g.num_nodes, g.edgeset_names, g.fwd, g.bwd,
                                       _native.MODE_RANDOM, seed=3, has_temporal=True)
    main = torch.cuda.current_stream(dev)
    gstream = torch.cuda.Stream(device=dev, priority=-1)
    # One tail stream per sampler: the tail (large-tree and padded kernels,
    # scans, compaction: ~250 us) is this step's critical path, and with a
    # shared tail stream consecutive tails would serialise.
    tstreams = [torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)]
    feats2 = [feats, torch.empty_like(feats)]
    S = max(d for d in range(1, min(steps, 10) + 1) if steps % d == 0)
    seeds_st = torch.zeros((S, B), dtype=torch.int64, device=dev)
    sts_st = torch.zeros((S, B), dtype=torch.int64, device=dev)

    def step_pipe(k):
        c = cc if k % 2 == 0 else cc_alt
        mm = c.sample_merged(seeds_st[k], sts_st[k], None, call_index=_native.CALL_INDEX_DEVICE, check=False,
                             tail_stream=tstreams[k % 2])
        gstream.wait_stream(tstreams[k % 2])
        with torch.cuda.stream(gstream):
            off = mm.node_offsets
            _native.check(_native.lib().dgfx_gather_rows_ranged(
                _native.ptr(table), n_a, FEAT_DIM * 4, _native.ptr(mm.node_ids), _native.elem_ptr(off, a * B),
                _native.elem_ptr(off, (a + 1) * B), int(mm.node_ids.numel()), _native.ptr(feats2[k % 2]),
                _native.stream_handle()))
        if not torch.cuda.is_current_stream_capturing():
            for t in (mm.node_ids, mm.node_offsets):
                t.record_stream(gstream)
        return mm

    def drain():
        cur = torch.cuda.current_stream(dev)
        for t in tstreams:
            cur.wait_stream(t)
        cur.wait_stream(gstream)

    seeds_st.copy_(seeds[:S])
    sts_st.copy_(sts[:S])
    for k in range(S):  # eager pass: streams, workspaces and size caches exist before capture
        step_pipe(k)
    drain()
    cc.check()
    cc_alt.check()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device=dev)
    cs.wait_stream(main)
    with torch.cuda.graph(graph, stream=cs):
        held = [step_pipe(k) for k in range(S)]  # outputs stay allocated for the replays
        drain()
    torch.cuda.synchronize(dev)

    def replay(r):
        seeds_st.copy_(seeds[8 + r * S:8 + (r + 1) * S], non_blocking=True)
        sts_st.copy_(sts[8 + r * S:8 + (r + 1) * S], non_blocking=True)
        graph.replay()

    for _ in range(3):
        replay(0)
    R = steps // S
    timed(replay, R, torch.cuda.synchronize, "hetero_pipelined")
    cc.check()
    cc_alt.check()
    ms = TIMING["hetero_pipelined"]["mean_ms"] / S  # whole timed region / K
    del graph, held, cc_alt, feats2
    out = {"workload": "heterogeneous temporal: A 736,389 / B 1,134,649 / C 8,740 / D 59,965 nodes; edges B->A "
                       "7,145,660, A->A 5,416,271, A->D 7,505,078, B->C 1,043,998 (Zipf 2.1); edge ts = "
                       "propagated A creation years; both directions, fanout [15,10]; 4096 A seeds, cutoff = seed "
                       "year; fp32 128-d A features",
           "value": round(B / (ms / 1e3), 1), "unit": "subgraphs/s", "ms_per_step": round(ms, 4),
           "step_time": "pipelined steps, up to 10 per CUDA-graph replay: whole timed region / K",
           "serial": {"value": round(B / (ms_serial / 1e3), 1), "ms_per_step": round(ms_serial, 4),
                      "note": "one stream, median per-step interval"},
           "nodes_per_step": nodes, "tree_positions": cc.tree_size, "graph_build_s": round(t_build, 2)}
    try:
        from oracle import oracle as O

        fwd, bwd = {}, {}
        for name, f, b in zip(g.edgeset_names, g.fwd, g.bwd):
            fwd[name] = (f.rowptr.cpu().numpy(), f.col.cpu().numpy(), None if f.ts is None else f.ts.cpu().numpy())
            bwd[name] = (b.rowptr.cpu().numpy(), b.col.cpu().numpy(), None if b.ts is None else b.ts.cpu().numpy())
        ref = O.available(ref=True)
        th = host_cores()
        s = O.OracleSampler.from_csr(g.num_nodes, g.nodeset_names, g.edgeset_names, fwd, plan, mode=O.MODE_RANDOM,
                                     num_threads=th, seed=99, temporal=True, ref=ref, csr_bwd=bwd)
        host_tab = table.cpu().numpy()
        seeds_h = seeds.cpu().numpy()
        sts_h = sts.cpu().numpy()
        done, t_tot, i = 0, 0.0, 0
        while t_tot < 10.0:
            t1 = time.perf_counter()
            nc, _, nodes_h, _, _ = s.sample_raw(seeds_h[i % nb], sts_h[i % nb], threads=th)
            off = 0
            for row in nc:  # per sample, node sets in order: gather A's rows
                lo = off + int(row[:a].sum())
                _ = host_tab[nodes_h[lo:lo + int(row[a])]]
                off += int(row.sum())
            t_tot += time.perf_counter() - t1
            done += B
            i += 1
        out["cpu_baseline"] = {"value": round(done / t_tot, 1), "unit": "subgraphs/s", "cores": th,
                               "kind": "reference" if ref else "port",
                               "sample": f"{done} seeds, topology + numpy gather of A features"}
        out["speedup_vs_cpu"] = round(out["value"] / out["cpu_baseline"]["value"], 1)
    except Exception as exc:  # noqa: BLE001
        out["cpu_baseline"] = {"unavailable": str(exc)}
    return out


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU sampler on the host cores.
# ---------------------------------------------------------------------------
def _chain_plan(nodeset, edgeset, widths):
    """A forward chain plan (root -hop_width[0]-> ... ) as plain objects with
    the SamplingPlan field names, so the reference arm imports nothing from
    the library."""
    from types import SimpleNamespace

    node = SimpleNamespace(nodeset=nodeset, children=[])
    for w in reversed(widths):
        node = SimpleNamespace(nodeset=nodeset, children=[
            SimpleNamespace(edgeset=edgeset, reversed=False, hop_width=int(w), node=node)])
    return SimpleNamespace(root=node, with_replacement=False)


# The large workload's generator parameters (the same GraphSpec as
# distributed_graph_flow_b200.synth.LARGE_SHARDED), repeated here so the
# reference arm does not import the library.
LARGE_NODES, LARGE_EDGES, LARGE_ALPHA, LARGE_MAX_DEG, LARGE_SEED = 111_059_956, 1_615_685_872, 2.0, 20_000, 4


def reference_arm(args, rank, world):
    """The reference's own CPU sampler on the host cores, on rank 0 only.

    Nothing here touches the GPU or loads the library: the graph, the seeds
    and the feature table come from the host restatement of the seeded
    generators (oracle/synth_cpu.h; the same graph, seeds and features as
    the device arm), the adjacency index is built by the reference's own
    AdjacencyIndex::CreateFromEdgeList (oracle/_ref, compiled from the
    reference's unmodified in_memory_sampler.cc; one call per source range
    on all host cores, concatenated), and each step samples one batch of
    8192 seeds with the reference's per-node samplers under the restated
    SampleBuilder / Sampler::Sample driver, then gathers every sampled
    node's feature row with numpy per sample (add_features_to_samples).
    Setup is untimed; W warm-up and K timed steps follow."""
    if rank != 0:
        return None
    from oracle import oracle as O

    cores = host_cores()
    ref = O.available(ref=True)
    scale = args.scale
    n = max(1000, int(LARGE_NODES * scale)) if scale != 1.0 else LARGE_NODES
    E = int(LARGE_EDGES * scale) if scale != 1.0 else LARGE_EDGES
    avail = host_mem_gb()
    # Index (8 B per edge + 8 B per node) + build transients (~16 B per edge)
    # + the bf16 feature table.
    need_gb = (24 * E + 8 * n) / 1e9 + n * FEAT_DIM * 2 / 1e9 + 8
    base = {"impl": "reference", "metric": "sampled subgraphs/sec", "unit": "subgraphs/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int64 ids / bf16 features",
            "data": "synthetic (the device arm's seeded graph, seeds and features, generated on the host)",
            "config": large_config(args, world)}
    if avail < need_gb:
        return dict(base, unavailable=f"host memory: the reference index and feature table need ~{need_gb:.0f} GB, "
                                      f"{avail:.0f} GB available")
    plan = _chain_plan("paper", "cites", FANOUT)
    t0 = time.perf_counter()
    s = O.OracleSampler.from_synth(n, E, LARGE_ALPHA, LARGE_MAX_DEG, LARGE_SEED, plan, mode=O.MODE_RANDOM,
                                   num_threads=cores, seed=99, ref=ref, build_threads=cores)
    t_index = time.perf_counter() - t0
    t0 = time.perf_counter()
    table = O.synth_normal_features(0, n, FEAT_DIM, LARGE_SEED + 100, bf16=True, threads=cores)
    t_feat = time.perf_counter() - t0
    W, K = args.warmup, args.steps
    seeds = O.synth_uniform_int((W + K) * B_SEEDS, 0, n, 77, 5, threads=cores).reshape(W + K, B_SEEDS)

    def step(batch):
        nc, _, nodes, _, _ = s.sample_raw(batch, threads=cores)
        off = 0
        for c in nc[:, 0]:
            _ = table[nodes[off:off + c]]
            off += c

    for i in range(W):
        step(seeds[i])
    per = []
    for i in range(K):
        t1 = time.perf_counter()
        step(seeds[W + i])
        per.append(time.perf_counter() - t1)
    ms = statistics.median(per) * 1e3
    rate = B_SEEDS / (ms / 1e3)
    return dict(base, value=round(rate, 1), ms_per_step=round(ms, 3),
                cpu_baseline={"value": round(rate, 1), "unit": "subgraphs/s", "cores": cores,
                              "kind": "reference" if ref else "port",
                              "sample": f"{K} timed batches of {B_SEEDS} seeds (median), after {W} warm-up; "
                                        f"topology by the reference's compiled samplers on {cores} threads + "
                                        f"numpy feature gather per sample"},
                e2e={"value": round(rate, 1), "unit": "subgraphs/s", "h2d_bytes_per_step": 0,
                     "d2h_bytes_per_step": 0},
                setup={"index_build_s": round(t_index, 1), "feature_table_s": round(t_feat, 1),
                       "index": "reference AdjacencyIndex::CreateFromEdgeList per source range" if ref else
                                "restated CreateFromEdgeList per source range",
                       "host_mem_available_gb": round(avail, 1)})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="dgfx", choices=["dgfx", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the SpMM / temporal sub-benchmarks")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--scale", type=float, default=1.0, help="shrink the workload (profiling / debugging only)")
    ap.add_argument("--only", default=None, choices=["large", "spmm", "temporal", "hetero", "sage", "gat", "negatives", "idmap"],
                    help="run one workload and skip the rest (profiling)")
    ap.add_argument("--halo", default="exchange", choices=["exchange", "p2p", "nccl"],
                    help="feature halo: bulk peer exchange (default), direct peer loads, or NCCL all-to-all")
    ap.add_argument("--halo-cache", type=float, default=0.5,
                    help="N > 1 with the bulk exchange: fraction of nodes (most in-edges first) whose feature rows "
                         "every GPU keeps a read-only copy of (0 disables; 0.5 = 14 GB per GPU on the 1.6B-edge "
                         "graph, of 180 GB)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="run each step's feature gather on the sampling stream (no pipelining)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="large sharded steps: issue every step from the host instead of replaying "
                         f"up to {GRAPH_STEPS} captured steps per CUDA graph")
    ap.add_argument("--no-split", dest="split", action="store_false",
                    help="overlapped steps: run each sampling call on one stream (no second sampler handle)")
    ap.add_argument("--minimal", action="store_true",
                    help="timed steps only: no e2e leg, launch count or CPU baseline (for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # Rank 0 alone times the reference's CPU sampler; other ranks exit.
        # No GPU, torch or library code runs in this arm.
        if rank == 0:
            print(json.dumps(reference_arm(args, rank, world)), flush=True)
        return

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    if args.only in ("spmm", "temporal", "hetero", "sage", "gat", "negatives", "idmap"):
        # Single sub-benchmark (used for focused profiler captures).
        fn = {"spmm": bench_spmm, "temporal": bench_temporal, "hetero": bench_hetero, "sage": bench_sage,
              "gat": bench_gat, "negatives": bench_rw_negatives, "idmap": bench_id_map}[args.only]
        print(json.dumps(fn(dev, args.steps, args.scale)), flush=True)
        return

    res, ctx = bench_large(args, rank, world, dev)
    spec, index, table, cc, plan, seeds, W, sharded = ctx
    if rank == 0 and world == 1 and args.only is None:
        if not args.no_cpu:
            table_host = None
            if host_mem_gb() > 80:
                table_host = table.cpu().view(torch.int16).numpy()
            try:
                from distributed_graph_flow_b200 import _native
                from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

                first = ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None],
                                                  _native.MODE_FIRST, seed=1234)
                rate, cores, kind, sample, par = cpu_large_baseline(index, table_host, spec.num_nodes, plan,
                                                                    seeds.cpu().numpy(), budget_s=15.0,
                                                                    parity=(first, seeds[W]))
                del first
                res["cpu_baseline"] = {"value": round(rate, 1), "unit": "subgraphs/s", "cores": cores, "kind": kind,
                                       "sample": json.dumps(sample)}
                res["parity"] = {"large_sharded": par}
            except Exception as exc:  # noqa: BLE001
                res["cpu_baseline"] = {"unavailable": str(exc)}
            del table_host
    # Peer-mapped partitions are unmapped and freed on every rank together.
    from distributed_graph_flow_b200 import driver as _driver

    if isinstance(sharded.features, _driver.PeerFeatures):
        sharded.features.close()
    del ctx, index, table, cc, sharded
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and args.only is None:
        if not args.no_extras:
            # Each sub-benchmark reports its own failure; the headline line
            # is printed regardless.
            legs = [("spmm", lambda: bench_spmm(dev, max(5, args.steps // 2))),
                    ("temporal_169k", lambda: bench_temporal(dev, args.steps)),
                    ("hetero_temporal", lambda: bench_hetero(dev, args.steps)),
                    ("sage_mean_2m", lambda: bench_sage(dev, args.steps)),
                    ("gat_attention_2m", lambda: bench_gat(dev, args.steps)),
                    ("rw_negatives_169k", lambda: bench_rw_negatives(dev, args.steps)),
                    ("gf_id_map_products", lambda: bench_id_map(dev, args.steps))]
            for key, fn in legs:
                try:
                    res[key] = fn()
                except Exception as exc:  # noqa: BLE001
                    res[key] = {"error": f"{type(exc).__name__}: {exc}"}
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
