#!/usr/bin/env python
"""bench.py -- FRNN throughput on the benchmark workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl engine|reference]
                    [--config C]

Workload (default ``--config 2``, the headline configuration): D=3, N=1,000,000
points from a 64-component Gaussian mixture (sigma=0.02), K=32, radius
calibrated for 24 mean in-radius neighbours, self-query.  One step = one full
search (grid build + neighbour search + results in the reference layout) of
one cloud.

Multi-GPU (one process per GPU under torchrun), ``--mode strong`` (default):
one cloud, its queries sharded over the ranks by the engine's own NCCL path
(frnn_search_sharded: rank 0 plans and builds the grid once and broadcasts the
built structure; every rank searches the queries of one work-balanced range of
original indices and its copy engines write that range's [K, rows] block
straight into rank 0's result buffers over NVLink -- all inside every step);
``value`` = N / max-over-ranks step time, ``shard`` reports every rank's stage
times and bytes.  ``--mode weak``: every rank
searches its own cloud -- replica ``rank`` of the configuration's
distribution -- with no data-path collective; ``value`` = all ranks'
queries / max-over-ranks step time.

Timing: W untimed warm-up steps, then exactly K timed steps, bracketed by a
barrier and torch.cuda.synchronize; each step is timed with CUDA events on the
engine's stream (the legacy default stream, which is also torch's current
stream); the L2 is flushed (a 512 MB buffer is overwritten) before every timed
step.  ``e2e`` times the same search through the host-buffer entry point
(pinned input copied in, all results copied out, every step).

The reference arm (``--impl reference``) runs the reference engine compiled
from its own sources for sm_100a (oracle/_ref/libfrnn_ref.so) through its
FRNNEngine.search_gpu on the same cloud, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "pure_cuda-c-_frnn_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

from frnn_cuda import datagen  # noqa: E402

L2_FLUSH_BYTES = 512 << 20
METRIC = "FRNN queries/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--n", type=int, default=None,
                    help="points (default: the configuration's own N; a smaller cloud gets a radius "
                         "calibrated for the same mean neighbour count) -- for small profiling cases")
    ap.add_argument("--k", type=int, default=None,
                    help="neighbours per query (default: the configuration's K) -- for small profiling "
                         "cases of other kernels")
    ap.add_argument("--shard-chunks", type=int, default=1,
                    help="strong mode: chunks per rank's slice, each sent while the next is searched")
    ap.add_argument("--shard-comm-priority", type=int, default=0, choices=[0, 1],
                    help="strong mode: 1 gives the gather's stream the highest priority")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per_config sweep over all five configurations (N=1 only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--mode", choices=["weak", "strong"], default="strong",
                    help="strong (default): one cloud, queries sharded over the ranks by the "
                         "engine's NCCL path (root builds once, broadcast, slice search, gather "
                         "to rank 0, all inside every step); weak: every rank searches its own "
                         "cloud with no data-path collective")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            j = json.load(f)
        return (float(j["hbm_gbs"]), float(j.get("bf16_tflops", 1590.0)),
                float(j.get("bf16_tflops_sustained", 1400.0)), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU, sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_uuid(torch, dev: int) -> str:
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return str(dev)


def time_steps(torch, fn, steps, flush):
    """Per-step device time (ms) of fn with an L2 flush before each step."""
    total = 0.0
    for _ in range(steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    return total / steps


def step_times(torch, fn, steps, flush):
    """Device time (ms) of each of ``steps`` calls of fn, L2 flushed before each."""
    out = []
    for _ in range(steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b))
    return out


def workload(cfg: int, n: int | None):
    """(config, points (N, D), radius) of a configuration, at its own size or n.

    The min-max normalised clouds (configurations 3 and 4) are clipped below
    1.0: the reference's first-coordinate grid drops points at 1.0
    (insert_points.cu:74-87) and its search then reads sorted slots that no
    point filled (find_nbrs.cu:254-256), which is undefined.  Clipping moves at
    most one point per coordinate by 1e-6 and leaves every measured time as it
    is; both arms search the same clipped cloud."""
    c = datagen.config(cfg)
    if n is None or n == c.N:
        pts, r = datagen.generate(c.kind, c.N, c.D, seed=datagen.SEED), c.radius
    else:
        pts, r = datagen.cloud(cfg, n)
    if c.kind.startswith("lowrank"):
        pts = np.minimum(pts, np.float32(0.999999))
    return c, pts, r


def config_dict(c, N: int, r: float, K: int | None = None) -> dict:
    """The ``config`` block: identical in both arms for the same workload."""
    K = K or c.K
    name = c.name + ("" if N == c.N else f"_n{N}") + ("" if K == c.K else f"_k{K}")
    return {"workload": name, "describe": c.describe, "N": N, "D": c.D, "K": K, "radius": r,
            "l2": "flushed before every timed step"}


def tc_filter_flops(N: int, D: int, symmetric: bool) -> float:
    """Flops the tensor-core filter must do: 2D per (query, point) pair, over
    all N^2 pairs, or over the N(N+1)/2 unordered pairs when a whole
    self-search filters each pair of tiles once (FRNN_OPT_TC_SYMMETRIC, the
    default; a sharded search filters its query tiles against all points)."""
    return float(N) * (N + 1) * D if symmetric else 2.0 * N * N * D


def search_roofline(N: int, D: int, K: int, cells: int, path: str, ms: float,
                    symmetric: bool = False) -> dict:
    """Whole-search roofline: the compulsory bytes B_alg = 4N(3D + 4 + 2K) + 12C
    of a grid search against HBM, or the tensor-core filter's flops
    (tc_filter_flops) against the sustained bf16 peak."""
    hbm, _, bf16_sus, src = measured_peaks()
    t = ms / 1e3
    if path == "brute_tc":
        f = tc_filter_flops(N, D, symmetric)
        return {"bound": "tensor", "alg_flops": f, "achieved": f / t / 1e12, "peak": bf16_sus,
                "unit": "TFLOP/s", "frac": f / t / 1e12 / bf16_sus, "peak_source": src + " (bf16 sustained)"}
    b = 4 * N * (3 * D + 4 + 2 * K) + 12 * cells
    return {"bound": "hbm", "alg_bytes": int(b), "achieved": b / t / 1e9, "peak": hbm, "unit": "GB/s",
            "frac": b / t / 1e9 / hbm, "peak_source": src}


def per_config_engine(torch, dev, flush, steps: int = 5, warmup: int = 3) -> dict:
    """Every configuration at full size on one GPU: median of ``steps`` timed
    searches (L2 flushed before each), per-stage times and the roofline."""
    import frnn_cuda
    out = {}
    for cfg in sorted(datagen.CONFIGS):
        c, pts, r = workload(cfg, None)
        soa = datagen.soa(pts)
        del pts
        x = torch.from_numpy(soa).to(dev)
        eng = frnn_cuda.FRNNEngine(max_points=c.N, device=dev)
        step = lambda: eng.search_gpu(x.data_ptr(), c.N, c.D, c.K, r)  # noqa: E731
        for _ in range(warmup):
            step()
        n = steps if cfg != 5 else 3
        ms = step_times(torch, step, n, flush)
        eng.set_timing(True)
        flush.zero_()
        step()
        stage_ms = eng.stage_times()
        eng.set_timing(False)
        plan = eng.last_plan()
        med = statistics.median(ms)
        out[f"cfg{cfg}"] = {"workload": c.name, "steps": n, "ms_median": med, "ms": ms,
                            "queries_per_s": c.N / (med / 1e3), "stage_ms": stage_ms, "plan": plan,
                            "roofline": search_roofline(c.N, c.D, c.K, plan["cells"], plan["path"], med,
                                                        symmetric=True)}
        del eng, x
        torch.cuda.empty_cache()
    return out


def per_config_sharded(torch, dist, rank, world, dev, flush, a, steps: int = 5, warmup: int = 3) -> dict:
    """Every configuration at full size, sharded over the ranks (rank 0's
    cloud): median over ``steps`` of the max-over-ranks search time."""
    import frnn_cuda
    from frnn_cuda.sharded import nccl_shard
    nmax = max(datagen.config(c).N for c in datagen.CONFIGS)
    eng = frnn_cuda.FRNNEngine(max_points=nmax, device=dev)
    shard = nccl_shard(eng)
    shard.set_timeout(300.0)
    shard.set_option(shard.OPT_CHUNKS, a.shard_chunks)
    out = {}
    for cfg in sorted(datagen.CONFIGS):
        c = datagen.config(cfg)
        x = None
        if rank == 0:
            _, pts, r = workload(cfg, None)
            x = torch.from_numpy(datagen.soa(pts)).to(dev)
            del pts
        r = c.radius
        xp = x.data_ptr() if x is not None else 0
        step = lambda: shard.search(0, xp, c.N, c.D, c.K, r)  # noqa: E731
        for _ in range(warmup):
            step()
        n = steps if cfg != 5 else 3
        dist.barrier()
        ms = step_times(torch, step, n, flush)
        t = torch.tensor(ms, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = [float(v) for v in t.tolist()]
        med = statistics.median(ms)
        plan = eng.last_plan()
        out[f"cfg{cfg}"] = {"workload": c.name, "steps": n, "ms_median": med, "ms": ms,
                            "queries_per_s": c.N / (med / 1e3), "plan": plan,
                            "shard": shard.last_stats()}
        del x
        torch.cuda.empty_cache()
    shard.close()
    return out


def per_config_reference(torch, dev, flush) -> dict:
    """The reference engine on every configuration at full size (its own
    dispatch): median of 5 timed searches, 2 for configuration 5, whose brute
    force takes about 47 s per search on a B200."""
    import oracle
    out = {}
    for cfg in sorted(datagen.CONFIGS):
        c, pts, r = workload(cfg, None)
        soa = datagen.soa(pts)
        del pts
        x = torch.from_numpy(soa).to(dev)
        ref = oracle.RefEngine(c.N)
        step = lambda: ref.search_gpu(x.data_ptr(), c.N, c.D, c.K, r)  # noqa: E731
        warm, n = (1, 2) if cfg == 5 else (3, 5)
        for _ in range(warm):
            step()
        ms = step_times(torch, step, n, flush)
        ref.close()
        plan = oracle.ref_plan(c.N, c.D, c.K, r)
        med = statistics.median(ms)
        path = "brute_tc" if plan["path"].startswith("bf") and c.D > 32 else "grid"
        out[f"cfg{cfg}"] = {"workload": c.name, "steps": n, "ms_median": med, "ms": ms,
                            "queries_per_s": c.N / (med / 1e3), "ref_path": plan["path"],
                            "roofline": search_roofline(c.N, c.D, c.K, plan["cells"], path, med)}
        del x
        torch.cuda.empty_cache()
    return out


def cpu_baseline(soa: np.ndarray, K: int, r: float, budget_s: float = 12.0) -> dict:
    """The CPU oracle (exact grid search, OpenMP) on a bounded query sample,
    extrapolated to the whole self-query."""
    import oracle
    D, N = soa.shape
    rng = np.random.default_rng(99)
    one = np.zeros(1, np.int32)
    t0 = time.perf_counter()
    oracle.search_subset(soa, one, K, r)
    t_build = time.perf_counter() - t0            # grid build + one query
    nq = min(N, 4096)
    while True:
        q = rng.choice(N, nq, replace=False).astype(np.int32)
        t0 = time.perf_counter()
        oracle.search_subset(soa, q, K, r)
        t = time.perf_counter() - t0
        if t >= 1.0 or nq == N:
            break
        nq = min(N, int(nq * max(2.0, min(budget_s, 5.0) / max(t, 1e-3))))
    t_query = max(t - t_build, 1e-9) / nq
    total = t_build + t_query * N
    return {"value": N / total, "unit": "queries/s", "cores": oracle.max_threads(), "kind": "port",
            "sample": f"oracle (C++/OpenMP exact grid search) on {nq} seeded queries of the same "
                      f"cloud plus one grid build; extrapolated to all {N} queries"}


def run_engine_arm(a, torch, dist, rank, world, dev):
    import frnn_cuda
    strong = a.mode == "strong" and world > 1
    c, pts, r = workload(a.config, a.n)
    N, D, K = pts.shape[0], c.D, a.k or c.K
    if not strong and rank > 0:
        # weak: rank r searches replica r (its own sample of the same distribution)
        pts = datagen.generate(c.kind, N, D, seed=datagen.SEED, replica=rank)
        if c.kind.startswith("lowrank"):
            pts = np.minimum(pts, np.float32(0.999999))
    soa = datagen.soa(pts)
    x = torch.from_numpy(soa).to(dev)
    eng = frnn_cuda.FRNNEngine(max_points=N, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    shard = None
    if strong:
        from frnn_cuda.sharded import _DeviceArray, nccl_shard
        shard = nccl_shard(eng)
        shard.set_timeout(120.0)
        shard.set_option(shard.OPT_CHUNKS, a.shard_chunks)
        shard.set_option(shard.OPT_COMM_PRIORITY, a.shard_comm_priority)
        xp = x.data_ptr() if rank == 0 else 0
        step = lambda: shard.search(0, xp, N, D, K, r)  # noqa: E731
    else:
        step = lambda: eng.search_gpu(x.data_ptr(), N, D, K, r)  # noqa: E731

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_uuid(torch, dev))
    # keep the GPU loaded while nvidia-smi starts, so the clock samples
    # describe the state the timed steps run in
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n0 = eng.launch_count()
    ms = time_steps(torch, step, a.steps, flush)
    launches = eng.launch_count() - n0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()

    # per-stage device times, from separate instrumented steps
    eng.set_timing(True)
    stages, sh_stages = {}, {}
    for _ in range(5):
        flush.zero_()
        step()
        for k, v in eng.stage_times().items():
            stages.setdefault(k, []).append(v)
        if shard is not None:
            for k, v in shard.last_stats()["stage_ms"].items():
                sh_stages.setdefault(k, []).append(v)
    eng.set_timing(False)
    stage_ms = {k: statistics.median(v) for k, v in stages.items()}
    plan = eng.last_plan()
    shard_ranks = None
    if shard is not None:
        mine = dict(shard.last_stats(), stage_ms={k: statistics.median(v) for k, v in sh_stages.items()},
                    engine_stage_ms=stage_ms, rank=rank)
        shard_ranks = [None] * world
        dist.all_gather_object(shard_ranks, mine)

    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = (1 if strong else world) * N / (ms_max / 1e3)

    # end-to-end through the host-buffer entry point (pinned buffers)
    e2e = None
    if not a.no_e2e:
        h_in = torch.from_numpy(soa).pin_memory()
        h_idx = torch.empty((K, N), dtype=torch.int32).pin_memory()
        h_dst = torch.empty((K, N), dtype=torch.float32).pin_memory()
        hi, hx, hd = h_in.numpy(), h_idx.numpy(), h_dst.numpy()
        if strong:
            def e2e_step():
                # rank 0: pinned host cloud in, sharded search, results out
                if rank == 0:
                    x.copy_(h_in, non_blocking=True)
                pi, pd = step()
                if rank == 0:
                    h_idx.copy_(torch.as_tensor(_DeviceArray(pi, (K, N), "<i4"), device=dev))
                    h_dst.copy_(torch.as_tensor(_DeviceArray(pd, (K, N), "<f4"), device=dev))
        else:
            e2e_step = lambda: eng.search_soa_host(hi, K, r, hx, hd)  # noqa: E731
        for _ in range(2):
            e2e_step()
        if world > 1:
            dist.barrier()
        e2e_ms = time_steps(torch, e2e_step, max(3, min(a.steps, 10)), flush)
        et = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": (1 if strong else world) * N / (float(et.item()) / 1e3), "unit": "queries/s",
               "h2d_bytes_per_step": int(N * D * 4), "d2h_bytes_per_step": int(N * K * 8),
               "ms_per_step": float(et.item())}

    if shard is not None:
        shard.close()  # before the process group goes: NCCL resources of this rank
    per_cfg = None
    if strong and not a.no_per_config:
        del x
        torch.cuda.empty_cache()
        per_cfg = per_config_sharded(torch, dist, rank, world, dev, flush, a)
    if rank != 0:
        return None

    hbm, bf16, bf16_sus, peak_src = measured_peaks()
    # dominant kernel: the stage with the largest device time
    dom = max(stage_ms, key=stage_ms.get) if stage_ms else None
    roofline = None
    # the share of the queries rank 0 searched (per-query kernels scale with it)
    qf = shard_ranks[0]["rows"] / N if shard_ranks else 1.0
    if dom is not None:
        cells = plan["cells"]
        row = 16 if D == 3 else ((D + 3) // 4 * 4 if D <= 16 else 32) * 4
        alg = {
            # rows read once + K results written + cell starts read
            "search": N * row + N * K * 8 + 4 * (cells + 1),
            "unpermute": N * K * 8 * 2 + 4 * N,
            "scan": 12 * cells,
            "hash": N * D * 4 + N * 8 + 4 * N,
            "scatter": N * D * 4 + N * 8 + N * row + 4 * N,
            "bbox": N * min(D, 4) * 4,
            "brute": N * D * 4 + N * K * 8,
            # lists hold every in-radius key (mean = the calibrated target count)
            "collect": N * row + 4 * (cells + 1) + N * c.target * 8 + 4 * N,
            "emit": N * c.target * 8 + 8 * N + N * K * 8,
            # tensor-core brute force: prep reads the SoA cloud, writes fp16
            # tiles, fp32 rows and two terms per point; the re-rank reads each
            # query's candidate rows (mean = the calibrated target count) and
            # writes K results
            "tc_prep": N * D * 4 + N * ((D + 63) // 64 * 64) * 2 + N * ((D + 3) // 4 * 4) * 4 + 8 * N,
            "tc_rerank": N * c.target * (((D + 3) // 4 * 4) * 4 + 4) + N * K * 8,
            # the filter is a dense contraction over every unordered pair once
            # (tc_filter_flops); a sharded search on 2..8 ranks shares that
            # triangle equally between the ranks
            "tc_filter": (tc_filter_flops(N, D, True) / world if world <= 8 else 2.0 * N * N * D * qf)
                         if strong else tc_filter_flops(N, D, True),
        }[dom]
        if dom in ("search", "collect", "emit", "tc_rerank", "brute", "unpermute"):
            alg *= qf
        t = stage_ms[dom] / 1e3
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath):
            with open(tpath) as f:
                traffic = json.load(f).get(f"cfg{a.config}", {}).get(dom)
        if dom == "tc_filter":
            # a kernel of hundreds of ms inside the step: the sustained peak
            achieved = alg / t / 1e12
            roofline = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": bf16_sus,
                        "unit": "TFLOP/s", "frac": achieved / bf16_sus, "traffic": traffic,
                        "peak_source": peak_src + " (bf16 sustained; the filter runs fp16 inputs "
                                                  "with fp32 accumulation, same dense rate)",
                        "alg_flops": alg, "kernel_ms": stage_ms[dom]}
        else:
            achieved = alg / t / 1e9
            roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm,
                        "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic,
                        "peak_source": peak_src, "alg_bytes": int(alg), "kernel_ms": stage_ms[dom]}
    b_alg = 4 * N * (3 * D + 4 + 2 * K) + 12 * plan["cells"]
    line = {
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": ("synthetic (seeded generator, seed 1234; rank 0's cloud, sharded)" if strong else
                 "synthetic (seeded generator, seed 1234; rank r draws replica r of the same distribution)"),
        "config": config_dict(c, N, r, K),
        "parallelism": (f"one cloud, queries sharded over {world} ranks by the engine's NCCL path: "
                        f"rank 0 builds once and broadcasts the built structure, every rank searches "
                        f"a work-balanced range of original query indices, and the copy engines move "
                        f"each range's results into rank 0's buffers over NVLink -- all in every "
                        f"step") if strong
                       else f"independent clouds x{world}",
        "queries_per_gpu": N // world if strong else N,
        "shard_options": {"chunks": a.shard_chunks, "comm_priority": a.shard_comm_priority} if strong else None,
        "latency_ms": ms_max,
        "pipeline": {"b_alg_bytes": int(b_alg), "b_alg_gbs": b_alg / (ms_max / 1e3) / 1e9,
                     "b_alg_frac": b_alg / (ms_max / 1e3) / 1e9 / hbm, "plan": plan,
                     "stage_ms": stage_ms},
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if shard_ranks:
        # per rank: device ms of each protocol stage and the bytes it moved;
        # the limiting collective is the slower of the broadcast and the gather
        # (the gather's time runs from the start of the rank's search to the
        # end of its last copy into rank 0's buffers)
        root = shard_ranks[0]["stage_ms"]
        coll = {k: root.get(k, 0.0) for k in ("broadcast", "gather")}
        line["shard"] = {"ranks": shard_ranks, "limiting_collective": max(coll, key=coll.get),
                         "collective_ms": coll,
                         "search_ms_max": max(r["stage_ms"].get("search", 0.0) for r in shard_ranks),
                         "search_ms_min": min(r["stage_ms"].get("search", 0.0) for r in shard_ranks)}
    if world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(soa, K, r)
    if world == 1 and not a.no_per_config:
        del x
        torch.cuda.empty_cache()
        line["per_config"] = per_config_engine(torch, dev, flush)
    if per_cfg is not None:
        line["per_config"] = per_cfg
    return line


def run_reference_arm(a, torch, dev):
    import oracle
    if not os.path.exists(oracle.REF_SO):
        return {"impl": "reference", "unavailable": "oracle/_ref/libfrnn_ref.so was not built"}
    c, pts, r = workload(a.config, a.n)
    N, D, K = pts.shape[0], c.D, a.k or c.K
    soa = datagen.soa(pts)
    x = torch.from_numpy(soa).to(dev)
    ref = oracle.RefEngine(N)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    step = lambda: ref.search_gpu(x.data_ptr(), N, D, K, r)  # noqa: E731
    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_uuid(torch, dev))
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        step()
    torch.cuda.synchronize()
    ms = time_steps(torch, step, a.steps, flush)
    clocks = sampler.stop()
    ref.close()
    value = N / (ms / 1e3)
    return {
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator, seed 1234)",
        "impl": "reference",
        "config": config_dict(c, N, r, K),
        "latency_ms": ms,
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": 1, "kind": "reference",
                         "sample": "the reference FRNNEngine.search_gpu, compiled from its own "
                                   "sources for sm_100a (oracle/_ref), full workload on GPU 0 "
                                   "(the reference has no CPU implementation of the path)"},
        "clocks": clocks,
    }


def main():
    a = parse()
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if a.impl == "reference":
        if rank != 0:
            return 0
        line = run_reference_arm(a, torch, local)
        if world == 1 and not a.no_per_config and "unavailable" not in line:
            flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=local)
            line["per_config"] = per_config_reference(torch, local, flush)
        print(json.dumps(line), flush=True)
        return 0
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        line = run_engine_arm(a, torch, dist, rank, world, local)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
