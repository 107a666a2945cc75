"""Benchmark harness with the reference's sweep conventions.

The reference times its engine with Tests/scripts/benchmark_vs_libfrnn.py:
a sweep over D x N cells (environment N_SWEEP, D_SWEEP, EXTRA_CELLS), K = 16,
seed 1234, clouds either uniform in [0,1)^D or low rank (DIST, INTRINSIC,
LOWRANK_NOISE), the radius analytic for uniform clouds and bisected on a
256-query sample otherwise, 20 warm-up and 10 timed calls of search_gpu with
the device synchronised around each, the median in ms, and a JSON file keyed
``D{D}_N{N}`` with fields R, dist, radius_mode, latency_ms, peak_mb and
libfrnn_gpu_ms (benchmark_vs_libfrnn.py:34-327).  This module restates those
conventions so that results of this engine land in the same JSON shape and
existing plotting and comparison scripts keep working:

    python -m frnn_cuda.harness [--out results.json]

The generators, the radius rules and the timing are the reference script's
(restated here, not imported); the cloud is the same for the same seed, so
numbers are comparable cell by cell.  ``libfrnn_gpu_ms`` is null: the xju2
libFRNN baseline is not part of this engine.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import time
from typing import Callable, Iterable

import numpy as np

K = 16
SEED = 1234
WARMUP = 20
TRIALS = 10
DEFAULT_N_SWEEP = (200000, 500000, 750000, 1000000, 1250000, 1500000)
DEFAULT_D_SWEEP = (3, 12, 16)


def settings(env=None) -> dict:
    """The sweep settings, from the same environment variables as the
    reference script (benchmark_vs_libfrnn.py:34-46)."""
    env = os.environ if env is None else env
    n_sweep = [int(n) for n in env.get("N_SWEEP", ",".join(map(str, DEFAULT_N_SWEEP))).split(",") if n.strip()]
    d_sweep = [int(d) for d in env.get("D_SWEEP", ",".join(map(str, DEFAULT_D_SWEEP))).split(",") if d.strip()]
    extra = [tuple(int(x) for x in c.split(":")) for c in env.get("EXTRA_CELLS", "").split(",") if c.strip()]
    cells = [(d, n) for d in d_sweep for n in n_sweep]
    cells += [c for c in extra if c not in cells]
    dist = env.get("DIST", "lowrank").lower()
    if dist not in ("uniform", "lowrank"):
        raise ValueError(f"unknown DIST={dist!r} (expected uniform|lowrank)")
    return {"cells": cells, "dist": dist, "intrinsic": int(env.get("INTRINSIC", "3")),
            "noise": float(env.get("LOWRANK_NOISE", "0.02"))}


def gen_points(N: int, D: int, seed: int = SEED, dist: str = "lowrank", intrinsic: int = 3,
               noise: float = 0.02) -> np.ndarray:
    """(N, D) float32 cloud (benchmark_vs_libfrnn.py:94-107): uniform in [0,1)^D,
    or a low-rank cloud -- uniform intrinsic coordinates mapped by a Gaussian
    embedding and a random rotation, plus isotropic noise -- min-max
    normalised to [0,1] per dimension.  Draw order follows the reference
    (legacy MT19937 stream), so the clouds are the same."""
    rng = np.random.RandomState(seed)
    if dist == "uniform" or intrinsic <= 0 or intrinsic >= D:
        return rng.rand(N, D).astype(np.float32)
    core = rng.rand(N, intrinsic)
    embed = rng.standard_normal((intrinsic, D))
    rot, _ = np.linalg.qr(rng.standard_normal((D, D)))
    pts = (core @ embed) @ rot + noise * rng.standard_normal((N, D))
    lo, hi = pts.min(0, keepdims=True), pts.max(0, keepdims=True)
    return ((pts - lo) / np.maximum(hi - lo, 1e-9)).astype(np.float32)


def radius_analytic(D: int, N: int, k: int = K) -> float:
    """Radius of a ball holding k expected points of a uniform unit cube,
    capped at 2 (benchmark_vs_libfrnn.py:84-91); 2 also when the reference's
    dense grid of ceil(1/r)^D cells would exceed 900,000 cells."""
    v = math.pi ** (D / 2) / math.gamma(D / 2 + 1)
    r = min((k / (N * v)) ** (1.0 / D), 2.0)
    if r < 1.0 and math.ceil(1.0 / r) ** D > 900_000:
        r = 2.0
    return round(r, 5)


def radius_calibrated(pts: np.ndarray, target: int = K, sample: int = 256, lo: float = 1e-4, hi: float = 2.0,
                      iters: int = 20) -> float:
    """Bisect r until the mean count of fp32 d^2 <= r^2 over a 256-query
    sample (legacy seed 0, without replacement) reaches target, 20 halvings
    of [1e-4, 2] (benchmark_vs_libfrnn.py:110-134)."""
    rng = np.random.RandomState(0)
    qi = rng.choice(len(pts), size=min(sample, len(pts)), replace=False)
    d2 = np.empty((len(qi), len(pts)), dtype=np.float32)
    for i, q in enumerate(pts[qi]):
        diff = pts - q
        d2[i] = (diff * diff).sum(axis=1)
    want = target * len(qi)
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        if int((d2 <= mid * mid).sum()) < want:
            lo = mid
        else:
            hi = mid
    return round(0.5 * (lo + hi), 6)


def timed_ms(fn: Callable[[], object], sync: Callable[[], None], warmup: int = WARMUP,
             trials: int = TRIALS) -> float:
    """Median wall time in ms of fn over `trials` calls after `warmup` calls,
    the device synchronised before and after each timed call
    (benchmark_vs_libfrnn.py:146-157)."""
    for _ in range(warmup):
        fn()
    sync()
    times = []
    for _ in range(trials):
        sync()
        t0 = time.perf_counter()
        fn()
        sync()
        times.append(time.perf_counter() - t0)
    return float(np.median(times)) * 1000.0


def run_cells(cells: Iterable[tuple], search: Callable[[np.ndarray, int, int, float], dict],
              dist: str = "lowrank", intrinsic: int = 3, noise: float = 0.02, log=print) -> dict:
    """One result per (D, N) cell: ``search(pts, N, D, R)`` returns
    {"latency_ms", "peak_mb"}; the result dict has the reference's JSON shape."""
    out = {}
    for D, N in cells:
        pts = gen_points(N, D, SEED, dist, intrinsic, noise)
        if dist == "uniform":
            R, mode = radius_analytic(D, N), "analytic"
        else:
            R, mode = radius_calibrated(pts), "calibrated"
        key = f"D{D}_N{N}"
        try:
            res = search(pts, N, D, R)
        except Exception as exc:  # reported like the reference script: the cell stays, latency null
            log(f"  [FRNN ERROR] {key}: {exc}")
            res = {"latency_ms": None, "peak_mb": None}
        out[key] = {"R": R, "dist": dist, "radius_mode": mode, "latency_ms": res.get("latency_ms"),
                    "peak_mb": res.get("peak_mb"), "libfrnn_gpu_ms": None}
        log(f"  {key}  R={R}  FRNN:{res.get('latency_ms')}ms")
    return out


def engine_search():
    """``search`` for run_cells backed by this engine on the current GPU: the
    SoA cloud on the device, FRNNEngine.search_gpu timed kernel-only (device
    pointer in, results on the device), device memory growth from NVML."""
    import torch
    import frnn_cuda

    try:
        import pynvml
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        used = lambda: pynvml.nvmlDeviceGetMemoryInfo(handle).used  # noqa: E731
    except Exception:  # NVML absent: no memory figure
        used = None

    def search(pts: np.ndarray, N: int, D: int, R: float) -> dict:
        x = torch.tensor(pts, device="cuda").T.contiguous()
        eng = frnn_cuda.FRNNEngine(max_points=N)
        torch.cuda.empty_cache()
        before = used() if used else None
        ms = timed_ms(lambda: eng.search_gpu(x.data_ptr(), N, D, K, R), torch.cuda.synchronize)
        peak = max(0, used() - before) / 1024 ** 2 if used else None
        eng.close()
        return {"latency_ms": ms, "peak_mb": None if peak is None else float(peak)}

    return search


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", default="vs_libfrnn_results.json", help="JSON results path")
    a = ap.parse_args(argv)
    st = settings()
    print(f"=== FRNN (B200 engine) | kernel-only | distribution: {st['dist']} ===")
    res = run_cells(st["cells"], engine_search(), st["dist"], st["intrinsic"], st["noise"])
    with open(a.out, "w") as f:
        json.dump(res, f, indent=2)
    print(f"-> {a.out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
