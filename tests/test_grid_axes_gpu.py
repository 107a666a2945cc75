"""The grid on principal axes (FRNN_OPT_GRID_AXES) against the oracle.

A grid on any orthonormal axes, with cells widened by the projection's
rounding bound, finds the same neighbours as the leading-coordinate grid; the
results must be bit-identical to the oracle's exact search for every D, data
kind and forced choice, and to each other."""

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


def run(frnn, soa, K, r, axes=None, path="grid"):
    D, N = soa.shape
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path(path)
    if axes is not None:
        eng.set_option(eng.OPT_GRID_AXES, axes)
    x = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    i, d = eng.get_results_arrays(N, K)
    return i, d, eng.last_plan()


@pytest.mark.parametrize("cfg,N", [(3, 60_000), (4, 60_000)])
def test_low_rank_clouds_pick_principal_axes(frnn, oracle_mod, cfg, N):
    c = datagen.config(cfg)
    pts, r = datagen.cloud(cfg, N)
    soa = datagen.soa(pts)
    i, d, plan = run(frnn, soa, c.K, r)
    assert plan["path"] == "grid" and plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search(soa, c.K, r)
    assert_bit_exact(i, d, oi, od, f"cfg{cfg} {plan}")


def test_isotropic_cloud_keeps_leading_coordinates(frnn, oracle_mod):
    N, D, K = 20000, 6, 16
    soa = datagen.soa(datagen.generate("uniform", N, D, seed=4))
    r = datagen.uniform_radius(N, 4, 20) * 1.5
    i, d, plan = run(frnn, soa, K, r)
    assert plan["axes"] == "leading", plan
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, "uniform D=6")


@pytest.mark.parametrize("D", [5, 6, 7, 8, 12, 16, 17, 24, 32])
@pytest.mark.parametrize("kind", ["lowrank4", "lowrank6", "mixture", "uniform"])
def test_forced_principal_axes(frnn, oracle_mod, D, kind):
    if kind == "lowrank6" and D < 6:
        pytest.skip("a rank-6 cloud needs D >= 6")
    N, K = 6000, 20
    pts = datagen.generate(kind, N, D, seed=D * 13 + len(kind))
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(np.ascontiguousarray(pts), 25, sample=512, seed=2)
    i, d, plan = run(frnn, soa, K, r, axes=2)
    # a cloud too spread for any grid (every axis <= 3 cells) is searched by
    # brute force instead
    assert plan["path"] == "brute" or plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, f"{kind} D={D} {plan}")


@pytest.mark.parametrize("K", [1, 33, 128])
def test_leading_and_principal_agree(frnn, K):
    N, D = 8000, 16
    pts = datagen.generate("lowrank6", N, D, seed=K)
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(np.ascontiguousarray(pts), 40, sample=512, seed=2)
    a = run(frnn, soa, K, r, axes=1)
    b = run(frnn, soa, K, r, axes=2)
    assert a[2]["axes"] == "leading" and b[2]["axes"] == "principal"
    assert_bit_exact(a[0], a[1], b[0], b[1], f"K={K}")


def test_principal_far_from_origin_and_scaled(frnn, oracle_mod):
    # the projection's rounding bound grows with |x - mu|: data offset and
    # scaled far from the unit box still searches exactly
    N, D, K = 6000, 10, 16
    pts = datagen.generate("lowrank4", N, D, seed=8).astype(np.float64)
    pts = (pts * 37.0 + 1.0e4).astype(np.float32)
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(np.ascontiguousarray(pts), 20, sample=512, seed=2)
    i, d, plan = run(frnn, soa, K, r, axes=2)
    assert plan["axes"] == "principal"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, "offset")


def test_principal_is_deterministic(frnn):
    c = datagen.config(4)
    pts, r = datagen.cloud(4, 30000)
    soa = datagen.soa(pts)
    a = run(frnn, soa, c.K, r)
    b = run(frnn, soa, c.K, r)
    assert a[2] == b[2]
    assert_bit_exact(a[0], a[1], b[0], b[1], "repeat")


def test_non_finite_in_trailing_dimension_rejected(frnn):
    N, D = 6000, 9
    pts = datagen.generate("lowrank4", N, D, seed=1)
    pts[77, 8] = np.nan
    soa = datagen.soa(pts)
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path("grid")
    eng.set_option(eng.OPT_GRID_AXES, 2)
    x = torch.from_numpy(soa).cuda()
    with pytest.raises(ValueError):
        eng.search_gpu(x.data_ptr(), N, D, 8, 0.1)


def test_option_rejects_unknown_mode(frnn):
    eng = frnn.FRNNEngine(max_points=10)
    with pytest.raises(ValueError):
        eng.set_option(eng.OPT_GRID_AXES, 3)


def test_list_search_option_rejects_unknown_mode(frnn):
    eng = frnn.FRNNEngine(max_points=10)
    with pytest.raises(ValueError):
        eng.set_option(eng.OPT_LIST_SEARCH, 3)


@pytest.mark.parametrize("kind,D,K,axes", [("uniform", 1, 16, 0), ("uniform", 2, 32, 0), ("mixture", 4, 20, 0),
                                           ("lowrank4", 8, 32, 2), ("lowrank4", 12, 8, 1), ("lowrank6", 16, 32, 2),
                                           ("mixture", 5, 16, 1), ("lowrank6", 24, 32, 2)])
@pytest.mark.parametrize("mode", ["AUTO", "ALWAYS", "NEVER"])
def test_list_search_modes_agree(frnn, oracle_mod, kind, D, K, axes, mode):
    # the list search (collect + emit) and the warp-cooperative search return
    # the same bits on leading-coordinate and principal-axis grids; queries
    # whose lists overflow go to the cooperative kernel in either mode
    N = 12000
    pts = datagen.generate(kind, N, D, seed=31 * D + K)
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(pts, 24, sample=512, seed=2)
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path("grid")
    eng.set_option(eng.OPT_GRID_AXES, axes)
    eng.set_option(eng.OPT_LIST_SEARCH, getattr(eng, "LIST_SEARCH_" + mode))
    x = torch.from_numpy(soa).cuda()
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    i, d = eng.get_results_arrays(N, K)
    assert eng.last_plan()["path"] == "grid"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, f"{kind} D={D} K={K} axes={axes} {mode}")
