"""Grids planned on the GPU (FRNN_OPT_DEVICE_PLAN), through the C ABI.

A blocking self-search with D <= 4 plans its grid inside the bounding-box
kernel and runs the build and search from that device-side plan, with no host
round trip in between; the reference reads the box back and plans on the host
(python_interface/frnn_engine.cu:64-86, 142-156).  The plan must be the host
planner's to the bit, and every branch the host takes after its plan -- no
useful grid (brute force), non-finite data (an error), the list search, the
cooperative search with direct or unpermuted output -- must come out the same.
Each case runs the same engine with the option on and off and compares results
bit for bit, the plan's cell count and axes, and the oracle.
"""

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

@pytest.fixture(scope="module")
def frnn():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    return frnn_cuda


def search(eng, soa, K, r, device_plan):
    D, N = soa.shape
    eng.set_option(eng.OPT_DEVICE_PLAN, device_plan)
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    idx, dist = eng.get_results_arrays(N, K)
    return idx, dist, eng.last_plan()


def both_ways(frnn, oracle_mod, soa, K, r, label, engine=None, want_path="grid"):
    D, N = soa.shape
    eng = engine or frnn.FRNNEngine(max_points=N)
    di, dd, dp = search(eng, soa, K, r, 1)
    hi, hd, hp = search(eng, soa, K, r, 0)
    assert dp == hp, f"{label}: device plan {dp} != host plan {hp}"
    assert dp["path"] == want_path, f"{label}: {dp}"
    assert_bit_exact(di, dd, hi, hd, f"{label}: device plan vs host plan")
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(di, dd, oi, od, f"{label}: device plan vs oracle")
    return eng


# (kind, N, D, K, radius scale): the kernels a D <= 4 grid search can take
CASES = [
    ("uniform", 60_000, 1, 8, 1.0),      # one axis, list search
    ("uniform", 60_000, 2, 16, 1.0),     # two axes, list search
    ("mixture", 100_000, 3, 32, 1.0),    # D = 3 collect + emit
    ("uniform", 50_000, 3, 64, 1.0),     # D = 3 cooperative search, direct output
    ("mixture", 40_000, 4, 32, 1.0),     # four axes, list search
    ("uniform", 40_000, 4, 40, 1.0),     # four axes, cooperative search
    ("mixture", 80_000, 3, 32, 2.2),     # many overflowing lists: the overflow pass
]


@pytest.mark.parametrize("kind,N,D,K,scale", CASES)
def test_device_plan_equals_host_plan(frnn, oracle_mod, kind, N, D, K, scale):
    pts = datagen.generate(kind, N, D, seed=7 * N + D)
    r = datagen.calibrate_radius(pts, 0.75 * min(K, 32), sample=256) * scale
    both_ways(frnn, oracle_mod, datagen.soa(pts), K, r, f"{kind} N={N} D={D} K={K}")


def test_unpermuted_output(frnn, oracle_mod):
    # D = 3, K > 32 with results larger than the direct-output limit: the
    # cooperative kernel writes cell order and the unpermute pass reorders
    pts = datagen.generate("uniform", 30_000, 3, seed=11)
    r = datagen.calibrate_radius(pts, 40, sample=256)
    eng = frnn.FRNNEngine(max_points=30_000)
    eng.set_option(eng.OPT_DIRECT_OUTPUT_MAX_BYTES, 0)
    both_ways(frnn, oracle_mod, datagen.soa(pts), 48, r, "unpermute", engine=eng)


def test_offset_and_scaled_clouds(frnn, oracle_mod):
    # boxes far from the origin and far from unit size: the planner's double
    # arithmetic (cell edge, slack, resolution) must round the same on the GPU
    base = datagen.generate("uniform", 40_000, 3, seed=3)
    for off, scale in [(1000.0, 1.0), (-3.5, 1e-3), (0.25, 4096.0)]:
        pts = (base * scale + off).astype(np.float32)
        r = datagen.calibrate_radius(pts, 12, sample=256)
        both_ways(frnn, oracle_mod, datagen.soa(pts), 16, r, f"offset {off} scale {scale}")


def test_no_useful_grid_falls_back_to_brute_force(frnn, oracle_mod):
    # N*N*D above the small-input rule, so the grid path is chosen, but the
    # radius spans a third of the box on every axis: the GPU's plan says "no
    # grid", every grid kernel returns at once, and the search runs brute force
    pts = datagen.generate("uniform", 12_000, 3, seed=5)
    both_ways(frnn, oracle_mod, datagen.soa(pts), 16, 0.45, "huge radius", want_path="brute")


def test_non_finite_points_rejected_then_usable(frnn, oracle_mod):
    pts = datagen.generate("uniform", 30_000, 3, seed=9)
    r = datagen.calibrate_radius(pts, 12, sample=256)
    bad = pts.copy()
    bad[1234, 1] = np.nan
    eng = frnn.FRNNEngine(max_points=30_000)
    for device_plan in (1, 0):
        # FRNN_ERR_INVALID_ARG surfaces as ValueError in the binding
        with pytest.raises(ValueError, match="NaN or Inf"):
            search(eng, datagen.soa(bad), 16, r, device_plan)
    both_ways(frnn, oracle_mod, datagen.soa(pts), 16, r, "after a rejected cloud", engine=eng)


def test_count_table_cleared_across_sizes(frnn, oracle_mod):
    # the cell tables are sized for the largest plan, and a kernel zeroes the
    # device plan's own count table: big, small, big again, different clouds,
    # one engine
    eng = frnn.FRNNEngine(max_points=200_000)
    for kind, N, seed in [("mixture", 200_000, 1), ("uniform", 20_000, 2), ("mixture", 150_000, 3),
                          ("uniform", 200_000, 4)]:
        pts = datagen.generate(kind, N, 3, seed=seed)
        r = datagen.calibrate_radius(pts, 20, sample=256)
        soa = datagen.soa(pts)
        idx, dist, plan = search(eng, soa, 32, r, 1)
        assert plan["path"] == "grid"
        oi, od, _ = oracle_mod.search(soa, 32, r)
        assert_bit_exact(idx, dist, oi, od, f"{kind} N={N} seed={seed}")


def test_scan_timeout_then_other_cloud(frnn, oracle_mod):
    # a scan that gives up ends the search with FRNN_ERR_TIMEOUT; the next
    # search, of a different cloud, on the same engine is exact
    pts, r = datagen.cloud(1, 60_000)
    eng = frnn.FRNNEngine(max_points=60_000)
    eng.set_option(eng.OPT_TEST_STALL, eng.TEST_STALL_SCAN)
    t = torch.from_numpy(np.ascontiguousarray(datagen.soa(pts))).cuda()
    with pytest.raises(frnn.FRNNError) as err:
        eng.search_gpu(t.data_ptr(), 60_000, 3, 16, r)
    assert err.value.status == 4, err.value
    eng.set_option(eng.OPT_TEST_STALL, eng.TEST_STALL_OFF)
    other = datagen.generate("mixture", 50_000, 3, seed=21)
    r2 = datagen.calibrate_radius(other, 16, sample=256)
    soa = datagen.soa(other)
    idx, dist, plan = search(eng, soa, 16, r2, 1)
    oi, od, _ = oracle_mod.search(soa, 16, r2)
    assert_bit_exact(idx, dist, oi, od, "after a scan timeout")
