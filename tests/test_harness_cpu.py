"""frnn_cuda.harness against the reference benchmark script's own functions.

tests/golden/harness/harness_golden.npz holds the outputs of the reference's
gen_points, calibrate_radius and radius_for on small seeded cases
(tests/golden/harness/make_harness_golden.py); the restated functions must reproduce
them exactly.  The sweep driver is run with a fake search to check the JSON
shape."""

import json
import os

import numpy as np
import pytest

from frnn_cuda import harness

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "harness", "harness_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.mark.parametrize("t", [0, 1, 2, 3])
def test_generator_matches_reference(gold, t):
    N, D, intrinsic, noise, uniform = gold[f"meta{t}"]
    pts = harness.gen_points(int(N), int(D), 1234, "uniform" if uniform else "lowrank", int(intrinsic), float(noise))
    assert pts.dtype == np.float32
    assert np.array_equal(pts, gold[f"pts{t}"])
    if not uniform:
        assert harness.radius_calibrated(pts, target=16) == float(gold[f"r{t}"])


def test_analytic_radius_matches_reference(gold):
    for D, N, r in gold["radius_for"]:
        assert harness.radius_analytic(int(D), int(N)) == r


def test_settings_follow_the_environment():
    st = harness.settings({"N_SWEEP": "1000,2000", "D_SWEEP": "3", "EXTRA_CELLS": "12:500,3:1000",
                           "DIST": "Uniform"})
    assert st["cells"] == [(3, 1000), (3, 2000), (12, 500)]
    assert st["dist"] == "uniform"
    with pytest.raises(ValueError):
        harness.settings({"DIST": "gaussian"})


def test_sweep_json_shape(tmp_path):
    calls = []

    def fake(pts, N, D, R):
        calls.append((N, D, R))
        if D == 12:
            raise RuntimeError("engine error")
        return {"latency_ms": 1.5, "peak_mb": 3.0}

    res = harness.run_cells([(3, 1500), (12, 800)], fake, "lowrank", 3, 0.02, log=lambda *a: None)
    assert list(res) == ["D3_N1500", "D12_N800"]
    assert set(res["D3_N1500"]) == {"R", "dist", "radius_mode", "latency_ms", "peak_mb", "libfrnn_gpu_ms"}
    assert res["D3_N1500"]["radius_mode"] == "calibrated" and res["D3_N1500"]["latency_ms"] == 1.5
    assert res["D12_N800"]["latency_ms"] is None
    json.dumps(res)


def test_timing_protocol_counts_calls():
    n = {"fn": 0, "sync": 0}
    ms = harness.timed_ms(lambda: n.__setitem__("fn", n["fn"] + 1), lambda: n.__setitem__("sync", n["sync"] + 1))
    assert n["fn"] == harness.WARMUP + harness.TRIALS
    assert n["sync"] == 1 + 2 * harness.TRIALS
    assert ms >= 0.0
