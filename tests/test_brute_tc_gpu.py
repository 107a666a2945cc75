"""Parity of the tensor-core brute force (FRNN_PATH_BRUTE_TC) with the oracle.

The tcgen05 fp16 filter only proposes candidates; every result comes from the
exact fp32 re-rank, so the arrays must be bit-identical to the oracle's exact
search (and to the SIMT brute force) on every input, including data whose
candidate lists overflow (identical points), data far from the origin (the
centring), data at tiny and huge scales (the power-of-two scaling) and
non-finite data (which the path hands to the SIMT kernel)."""

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


def run(frnn, soa, K, r, path="brute_tc"):
    D, N = soa.shape
    eng = frnn.FRNNEngine(max_points=N)
    if path is not None:
        eng.set_path(path)
    t = torch.from_numpy(np.ascontiguousarray(soa, dtype=np.float32)).cuda()
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    idx, dist = eng.get_results_arrays(N, K)
    return idx, dist, eng.last_plan()


def sphere(N, D, seed):
    return datagen.generate("sphere", N, D, seed=seed)


def radius_for(soa, target, seed=7):
    pts = np.ascontiguousarray(soa.T)
    return datagen.calibrate_radius(pts, target, sample=min(512, len(pts)), seed=seed)


@pytest.mark.parametrize("D", [33, 48, 64, 65, 100, 128])
@pytest.mark.parametrize("K", [1, 16, 128])
def test_dims_and_k(frnn, oracle_mod, D, K):
    N = 3000
    soa = datagen.soa(sphere(N, D, seed=D * 7 + K))
    r = radius_for(soa, 40)
    idx, dist, plan = run(frnn, soa, K, r)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"D={D} K={K}")


@pytest.mark.parametrize("N", [1, 2, 127, 128, 129, 255, 256, 257, 1000])
def test_tile_edges(frnn, oracle_mod, N):
    D, K = 128, 32
    soa = datagen.soa(sphere(N, D, seed=N))
    r = 1.2
    idx, dist, plan = run(frnn, soa, K, r)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"N={N}")


@pytest.mark.parametrize("D", [3, 8, 16, 32])
def test_low_dims_forced(frnn, oracle_mod, D):
    # the filter works for any D <= 128 (one 64-dimension slab); the re-rank
    # uses the D = 3 order for D = 3 and the chain otherwise
    N, K = 4000, 16
    soa = datagen.soa(datagen.generate("uniform", N, D, seed=D))
    r = radius_for(soa, 24)
    idx, dist, plan = run(frnn, soa, K, r)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"D={D}")


def test_cfg5_cloud_auto_dispatch(frnn, oracle_mod):
    c = datagen.config(5)
    pts, r = datagen.cloud(5, 12_000)
    soa = datagen.soa(pts)
    idx, dist, plan = run(frnn, soa, c.K, r, path=None)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, c.K, r)
    assert_bit_exact(idx, dist, oi, od, "cfg5 12K")


def test_matches_simt_bruteforce(frnn):
    N, D, K = 9000, 96, 64
    soa = datagen.soa(sphere(N, D, seed=5))
    r = radius_for(soa, 80)
    a = run(frnn, soa, K, r, path="brute_tc")
    b = run(frnn, soa, K, r, path="brute")
    assert a[2]["path"] == "brute_tc" and b[2]["path"] == "brute"
    assert_bit_exact(a[0], a[1], b[0], b[1], "tc vs simt")


def test_identical_points_overflow(frnn, oracle_mod):
    # every pair is in radius: all candidate lists overflow and the SIMT pass
    # answers every query
    N, D, K = 1500, 64, 128
    soa = np.full((D, N), 0.25, dtype=np.float32)
    idx, dist, plan = run(frnn, soa, K, 0.5)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, 0.5)
    assert_bit_exact(idx, dist, oi, od, "identical")


def test_dense_cluster_mixed_overflow(frnn, oracle_mod):
    # a tight cluster (lists overflow) beside spread points (lists fit)
    rng = np.random.default_rng(3)
    D, K = 40, 16
    spread = rng.standard_normal((2500, D)).astype(np.float32)
    cluster = (0.001 * rng.standard_normal((600, D))).astype(np.float32)
    pts = np.concatenate([spread[:1200], cluster, spread[1200:]])
    soa = datagen.soa(pts)
    idx, dist, plan = run(frnn, soa, K, 0.5)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, 0.5)
    assert_bit_exact(idx, dist, oi, od, "cluster")


@pytest.mark.parametrize("shift,scale", [(1000.0, 1.0), (-3.0e4, 1.0), (0.0, 1e-12), (0.0, 1e12),
                                         (7.5, 1e-3)])
def test_offset_and_scale(frnn, oracle_mod, shift, scale):
    N, D, K = 2500, 64, 32
    base = sphere(N, D, seed=11)
    pts = (base * np.float32(scale) + np.float32(shift)).astype(np.float32)
    soa = datagen.soa(pts)
    r = radius_for(soa, 30)
    idx, dist, plan = run(frnn, soa, K, r)
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"shift={shift} scale={scale} {plan}")


def test_duplicates_and_ties(frnn, oracle_mod):
    # repeated rows give exact distance ties; ranks fall back to the index
    rng = np.random.default_rng(9)
    D, K = 72, 20
    uniq = rng.random((700, D)).astype(np.float32)
    pts = uniq[rng.integers(0, 700, 2800)]
    soa = datagen.soa(pts)
    r = radius_for(soa, 30)
    idx, dist, plan = run(frnn, soa, K, r)
    assert plan["path"] == "brute_tc"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, "duplicates")


def test_non_finite_goes_to_simt(frnn, oracle_mod):
    N, D, K = 1200, 48, 8
    pts = sphere(N, D, seed=2)
    pts[5, 3] = np.inf
    pts[17, 0] = np.nan
    soa = datagen.soa(pts)
    idx, dist, plan = run(frnn, soa, K, 1.0)
    assert plan["path"] == "brute"
    oi, od, _ = oracle_mod.search(soa, K, 1.0)
    assert_bit_exact(idx, dist, oi, od, "non-finite")


def test_repeat_calls_reuse_engine(frnn, oracle_mod):
    # one engine, shapes growing and shrinking: scratch and lists are reused
    eng = frnn.FRNNEngine(max_points=5000)
    eng.set_path("brute_tc")
    for N, D, K in [(5000, 128, 64), (700, 40, 128), (3000, 64, 1), (5000, 128, 64)]:
        soa = datagen.soa(sphere(N, D, seed=N + D))
        r = radius_for(soa, 50)
        t = torch.from_numpy(soa).cuda()
        eng.search_gpu(t.data_ptr(), N, D, K, r)
        idx, dist = eng.get_results_arrays(N, K)
        oi, od, _ = oracle_mod.search(soa, K, r)
        assert_bit_exact(idx, dist, oi, od, f"N={N} D={D} K={K}")
