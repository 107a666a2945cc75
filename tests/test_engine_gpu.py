"""Parity of the CUDA engine with the CPU oracle, through the C ABI.

Every case compares the engine's SoA results with the oracle's exact search
on the same seeded input: both rank by (d2, index) with the same fp32
arithmetic, so the arrays must be bit-identical.  Paths are also forced one by
one (grid, brute force) to show that every path returns the same answer."""

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


def run_engine(frnn, soa, K, r, path=None, engine=None):
    D, N = soa.shape
    eng = engine or frnn.FRNNEngine(max_points=N)
    if path is not None:
        eng.set_path(path)
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    pi, pd = eng.search_gpu(t.data_ptr(), N, D, K, r)
    assert pi and pd
    idx, dist = eng.get_results_arrays(N, K)
    plan = eng.last_plan()
    return idx, dist, plan


# (config, reduced N) -- the five benchmark clouds at sizes the oracle finishes quickly
CASES = [(1, 20_000), (2, 40_000), (3, 20_000), (4, 20_000), (5, 3_000)]


@pytest.mark.parametrize("cfg,N", CASES)
def test_config_clouds_auto_path(frnn, oracle_mod, cfg, N):
    c = datagen.config(cfg)
    pts, r = datagen.cloud(cfg, N)
    soa = datagen.soa(pts)
    idx, dist, plan = run_engine(frnn, soa, c.K, r)
    oi, od, _ = oracle_mod.search(soa, c.K, r)
    assert_bit_exact(idx, dist, oi, od, f"cfg{cfg} {plan}")


@pytest.mark.parametrize("cfg,N", [(1, 6_000), (2, 8_000), (3, 6_000), (4, 6_000)])
@pytest.mark.parametrize("path", ["grid", "brute"])
def test_forced_paths_agree(frnn, oracle_mod, cfg, N, path):
    c = datagen.config(cfg)
    pts, r = datagen.cloud(cfg, N)
    soa = datagen.soa(pts)
    idx, dist, plan = run_engine(frnn, soa, c.K, r, path=path)
    assert plan["path"] == path
    oi, od, _ = oracle_mod.search(soa, c.K, r)
    assert_bit_exact(idx, dist, oi, od, f"cfg{cfg} {path}")


@pytest.mark.parametrize("D", [1, 2, 3, 4, 5, 7, 8, 12, 16, 17, 24, 32])
@pytest.mark.parametrize("K", [1, 16, 33])
def test_dimensions_grid(frnn, oracle_mod, D, K):
    N = 5000
    pts = datagen.generate("lowrank4" if D > 4 else "uniform", N, D, seed=D * 101 + K)
    soa = datagen.soa(pts)
    r = datagen.uniform_radius(N, min(D, 4), 20) * (1.5 if D > 4 else 1.0)
    idx, dist, plan = run_engine(frnn, soa, K, r, path="grid")
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"D={D} K={K} {plan}")


@pytest.mark.parametrize("D", [3, 33, 64, 128])
def test_bruteforce_high_dims(frnn, oracle_mod, D):
    N = 2000
    pts = datagen.generate("sphere", N, D, seed=D)
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(pts, 20, sample=256)
    idx, dist, plan = run_engine(frnn, soa, 128 if D == 128 else 40, r)
    oi, od, _ = oracle_mod.search(soa, 128 if D == 128 else 40, r)
    assert_bit_exact(idx, dist, oi, od, f"D={D} {plan}")


# ---- edge cases ------------------------------------------------------------------


def test_single_point(frnn, oracle_mod):
    soa = np.array([[0.5], [0.25], [0.75]], np.float32)
    idx, dist, _ = run_engine(frnn, soa, 4, 0.1)
    assert idx[:, 0].tolist() == [0, -1, -1, -1]
    assert dist[0, 0] == 0.0 and np.all(dist[1:, 0] == np.float32(0.1) * np.float32(0.1))


@pytest.mark.parametrize("path", ["grid", "brute"])
def test_duplicate_points_ties_break_by_index(frnn, oracle_mod, path):
    rng = np.random.default_rng(0)
    base = rng.random((300, 3)).astype(np.float32)
    pts = np.repeat(base, 40, axis=0)  # 40 copies of each point: ties at d2 = 0
    rng.shuffle(pts)
    soa = datagen.soa(pts)
    idx, dist, _ = run_engine(frnn, soa, 16, 0.05, path=path)
    oi, od, _ = oracle_mod.search(soa, 16, 0.05)
    assert_bit_exact(idx, dist, oi, od, "duplicates")
    # every slot is a duplicate at distance 0, lowest indices first
    assert np.all(dist == 0.0)


@pytest.mark.parametrize("K", [8, 16, 20, 32])
@pytest.mark.parametrize("path", ["grid", "brute"])
def test_lattice_ties_at_the_kth_distance(frnn, oracle_mod, K, path):
    # A lattice with spacing 2^-6: coordinates, differences and squared
    # distances are exact in fp32, so the 26 neighbours of an inner point sit at
    # exactly three distances (6, 12 and 8 of them) and the K-th slot (the
    # point itself is the first) falls inside a tie for K = 8, 16 and 20; ties
    # resolve to the smaller index.
    g = np.arange(16, dtype=np.float32) / 64.0
    pts = np.stack(np.meshgrid(g, g, g, indexing="ij"), axis=-1).reshape(-1, 3)
    pts = pts[np.random.default_rng(1).permutation(len(pts))]
    soa = datagen.soa(pts)
    r = 1.8 / 64.0
    idx, dist, _ = run_engine(frnn, soa, K, r, path=path)
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"lattice K={K}")
    # an inner point keeps itself and its K - 1 nearest lattice neighbours,
    # ties by index
    inner = np.flatnonzero(np.all((pts > 0) & (pts < g[-1]), axis=1))[0]
    d = ((pts - pts[inner]) ** 2).sum(axis=1)
    order = np.lexsort((np.arange(len(pts)), d))
    want = [int(j) for j in order if d[j] < np.float32(r) * np.float32(r)][:K]
    assert idx[:, inner].tolist() == want + [-1] * (K - len(want))


def test_all_points_identical(frnn, oracle_mod):
    soa = np.full((3, 3000), 0.3, np.float32)
    idx, dist, _ = run_engine(frnn, soa, 8, 0.01, path="grid")
    assert np.array_equal(idx, np.tile(np.arange(8, dtype=np.int32)[:, None], (1, 3000)))


def test_points_outside_unit_cube(frnn, oracle_mod):
    rng = np.random.default_rng(4)
    pts = (rng.standard_normal((30000, 3)) * 5.0 - 3.0).astype(np.float32)
    soa = datagen.soa(pts)
    r = 0.6
    idx, dist, plan = run_engine(frnn, soa, 12, r)
    oi, od, _ = oracle_mod.search(soa, 12, r)
    assert plan["path"] == "grid"
    assert_bit_exact(idx, dist, oi, od, "outside [0,1)")


def test_radius_covers_everything(frnn, oracle_mod):
    pts = datagen.generate("uniform", 3000, 3, seed=1)
    soa = datagen.soa(pts)
    idx, dist, _ = run_engine(frnn, soa, 32, 10.0)
    oi, od, _ = oracle_mod.search(soa, 32, 10.0)
    assert_bit_exact(idx, dist, oi, od, "huge radius")
    assert np.all(idx >= 0)


def test_tiny_radius_only_self(frnn, oracle_mod):
    pts = datagen.generate("uniform", 50000, 3, seed=2)
    soa = datagen.soa(pts)
    idx, dist, _ = run_engine(frnn, soa, 4, 1e-7)
    assert np.array_equal(idx[0], np.arange(50000, dtype=np.int32))
    assert np.all(idx[1:] == -1)


def test_ragged_sizes(frnn, oracle_mod):
    for N in (1, 2, 31, 127, 129, 4097):
        pts = datagen.generate("uniform", N, 3, seed=N)
        soa = datagen.soa(pts)
        for path in ("grid", "brute"):
            idx, dist, _ = run_engine(frnn, soa, 5, 0.3, path=path)
            oi, od, _ = oracle_mod.search(soa, 5, 0.3)
            assert_bit_exact(idx, dist, oi, od, f"N={N} {path}")


def test_max_k(frnn, oracle_mod):
    pts = datagen.generate("mixture", 20000, 3, seed=3)
    soa = datagen.soa(pts)
    for path in ("grid", "brute"):
        idx, dist, _ = run_engine(frnn, soa, 128, 0.03, path=path)
        oi, od, _ = oracle_mod.search(soa, 128, 0.03)
        assert_bit_exact(idx, dist, oi, od, f"K=128 {path}")


def test_engine_reuse_across_shapes(frnn, oracle_mod):
    eng = frnn.FRNNEngine(max_points=30000)
    for (N, D, K, seed) in [(30000, 3, 16, 1), (1000, 12, 64, 2), (20000, 2, 8, 3), (30000, 3, 32, 4)]:
        pts = datagen.generate("uniform", N, D, seed=seed)
        soa = datagen.soa(pts)
        r = datagen.uniform_radius(N, min(D, 4), 12)
        idx, dist, _ = run_engine(frnn, soa, K, r, engine=eng)
        oi, od, _ = oracle_mod.search(soa, K, r)
        assert_bit_exact(idx, dist, oi, od, f"reuse N={N} D={D}")


@pytest.mark.parametrize("D,K", [(3, 16), (3, 48), (2, 8), (4, 32)])
def test_points_changed_in_place_between_searches(frnn, oracle_mod, D, K):
    # One engine searches the same device buffer while its contents change
    # between calls (unchanged, moved, grown, shrunk, then a NaN): every call
    # plans its grid from that call's points, so each must match the oracle or
    # report the NaN, and a clean call after the NaN recovers.
    N = 20000
    base = datagen.generate("mixture", N, D, seed=D + K)
    r = datagen.calibrate_radius(base, 16, sample=512, seed=5)
    eng = frnn.FRNNEngine(max_points=N)
    x = torch.empty((D, N), dtype=torch.float32, device="cuda")
    for step, pts in enumerate([base, base, base + 0.3, base * 1.5, base * 0.7, base * 0.7]):
        soa = datagen.soa(pts.astype(np.float32))
        x.copy_(torch.from_numpy(soa))
        eng.search_gpu(x.data_ptr(), N, D, K, r)
        i, d = eng.get_results_arrays(N, K)
        oi, od, _ = oracle_mod.search(soa, K, r)
        assert_bit_exact(i, d, oi, od, f"step {step} D={D} K={K}")
        assert eng.last_plan()["path"] == "grid"
    x[0, 123] = float("nan")
    with pytest.raises(ValueError):
        eng.search_gpu(x.data_ptr(), N, D, K, r)
    x[0, 123] = 0.5
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    i, d = eng.get_results_arrays(N, K)
    oi, od, _ = oracle_mod.search(x.cpu().numpy(), K, r)
    assert_bit_exact(i, d, oi, od, "after the NaN")


# ---- the reference's host-path and results surface ------------------------------


def test_host_search_lists_row_major(frnn, oracle_mod):
    N, D, K = 4000, 3, 8
    pts = datagen.generate("uniform", N, D, seed=9)
    r = datagen.uniform_radius(N, D, 10)
    eng = frnn.FRNNEngine(max_points=N)
    idxs, dists = eng.search(pts.reshape(-1).tolist(), K, r)
    assert isinstance(idxs, list) and len(idxs) == N * K
    oi, od, _ = oracle_mod.search(datagen.soa(pts), K, r)
    assert np.array_equal(np.asarray(idxs, np.int32).reshape(N, K), oi.T)
    assert np.array_equal(np.asarray(dists, np.float32).reshape(N, K), od.T)
    # get_results returns the same results in SoA order
    gi, gd = eng.get_results(N, K)
    assert np.array_equal(np.asarray(gi, np.int32).reshape(K, N), oi)
    gi2, _ = eng.get_results(N, 3)  # first K' rows
    assert np.array_equal(np.asarray(gi2, np.int32).reshape(3, N), oi[:3])


def test_host_soa_path(frnn, oracle_mod):
    N, D, K = 5000, 16, 24
    pts = datagen.generate("lowrank6", N, D, seed=10)
    soa = datagen.soa(pts)
    r = 0.2
    eng = frnn.FRNNEngine(max_points=N)
    i, d = eng.search_soa_host(soa, K, r)
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, "host soa")


@pytest.mark.parametrize("N,K,r", [(300, 8, 0.2), (20011, 16, 0.03), (40000, 32, 0.02), (20000, 32, 0.08)])
def test_host_soa_d3(frnn, oracle_mod, N, K, r):
    # the D = 3 collect/emit path through the host-buffer entry point: both
    # emit widths, ragged sizes, and lists that overflow into the cooperative
    # pass (a few, most, nearly all); pinned and pageable outputs
    pts = datagen.generate("mixture", N, 3, seed=N)
    soa = datagen.soa(pts)
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path("grid")
    hi = torch.empty((K, N), dtype=torch.int32).pin_memory().numpy()
    hd = torch.empty((K, N), dtype=torch.float32).pin_memory().numpy()
    i, d = eng.search_soa_host(soa, K, r, hi, hd)
    assert eng.last_plan()["path"] == "grid"
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, f"host soa N={N} K={K}")
    i2, d2 = eng.search_soa_host(soa, K, r)
    assert np.array_equal(i2, i) and np.array_equal(d2.view(np.int32), d.view(np.int32))
    # the device-pointer entry point afterwards still returns the same rows
    x = torch.from_numpy(soa).cuda()
    eng.search_gpu(x.data_ptr(), N, 3, K, r)
    gi, gd = eng.get_results_arrays(N, K)
    assert np.array_equal(gi, i) and np.array_equal(gd.view(np.int32), d.view(np.int32))


# ---- errors are reported, not undefined -------------------------------------------


def test_argument_errors(frnn):
    eng = frnn.FRNNEngine(max_points=100)
    t = torch.rand(3 * 100, device="cuda")
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 101, 3, 4, 0.1)      # N > max_points
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 100, 3, 0, 0.1)      # K = 0
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 100, 3, 129, 0.1)    # K > 128
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 100, 129, 4, 0.1)    # D > 128
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 100, 3, 4, 0.0)      # r = 0
    with pytest.raises(ValueError):
        eng.search_gpu(t.data_ptr(), 100, 3, 4, float("nan"))
    host = np.zeros(300, np.float32)
    with pytest.raises(ValueError):
        eng.search_gpu(host.ctypes.data, 100, 3, 4, 0.1)  # not device memory
    with pytest.raises(frnn.FRNNError):
        eng.get_results(100, 4)                            # nothing searched yet
    bad = torch.rand(3 * 100, device="cuda")
    bad[17] = float("nan")
    eng.set_path("grid")
    with pytest.raises(ValueError):
        eng.search_gpu(bad.data_ptr(), 100, 3, 4, 0.1)    # non-finite coordinates
    # the engine stays usable after errors
    pi, pd = eng.search_gpu(t.data_ptr(), 100, 3, 4, 0.1)
    assert pi and pd


def test_search_is_deterministic(frnn):
    pts, r = datagen.cloud(2, 100_000)
    soa = datagen.soa(pts)
    a = run_engine(frnn, soa, 32, r)
    b = run_engine(frnn, soa, 32, r)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.parametrize("K", [8, 16, 32])
def test_dense_lists_overflow_to_cooperative_pass(frnn, oracle_mod, K):
    # D=3 with K <= 32 collects every in-radius key per query (64 or 128 of
    # them at most) and hands queries with more to the cooperative kernel:
    # a dense core (hundreds in radius) next to a sparse halo exercises both.
    rng = np.random.default_rng(K)
    core = (0.5 + 0.002 * rng.standard_normal((3000, 3))).astype(np.float32)
    halo = rng.random((20000, 3)).astype(np.float32)
    pts = np.concatenate([halo[:10000], core, halo[10000:]])
    soa = datagen.soa(pts)
    idx, dist, plan = run_engine(frnn, soa, K, 0.01, path="grid")
    oi, od, _ = oracle_mod.search(soa, K, 0.01)
    assert_bit_exact(idx, dist, oi, od, f"overflow K={K}")


@pytest.mark.parametrize("limit", [0, 1 << 40])
def test_d3_cooperative_unpermute_and_direct(frnn, oracle_mod, limit):
    # D = 3 with K > 32 runs the cooperative kernel; results go through the
    # unpermute pass when larger than FRNN_OPT_DIRECT_OUTPUT_MAX_BYTES
    c = datagen.config(2)
    pts, r = datagen.cloud(2, 30000)
    soa = datagen.soa(pts)
    eng = frnn.FRNNEngine(max_points=30000)
    eng.set_option(eng.OPT_DIRECT_OUTPUT_MAX_BYTES, limit)
    eng.set_timing(True)
    idx, dist, plan = run_engine(frnn, soa, 48, r, path="grid", engine=eng)
    assert ("unpermute" in eng.stage_times()) == (limit == 0)
    oi, od, _ = oracle_mod.search(soa, 48, r)
    assert_bit_exact(idx, dist, oi, od, f"K=48 limit={limit}")


def test_fresh_engines_on_reused_memory(frnn, oracle_mod):
    """Engines created one after another get device memory that earlier
    engines freed.  The prefix scan tags its look-back status words with a
    per-engine epoch that starts at 1 in every engine, so a status buffer that
    reuses an earlier engine's memory must be cleared first, or the new
    engine's first scan reads that engine's sums as its own.  Two clouds with
    the same grid size but different cell counts, searched alternately by
    fresh engines, must each stay exact."""
    N, K = 150_000, 16
    clouds = []
    for seed in (11, 12):
        pts = np.random.default_rng(seed).random((N, 3), dtype=np.float64).astype(np.float32)
        soa = datagen.soa(pts)
        r = datagen.uniform_radius(N, 3, K)
        oi, od, _ = oracle_mod.search(soa, K, r)
        clouds.append((soa, r, oi, od))
    for it in range(6):
        soa, r, oi, od = clouds[it % 2]
        idx, dist, plan = run_engine(frnn, soa, K, r)
        assert plan["path"] == "grid"
        assert_bit_exact(idx, dist, oi, od, f"fresh engine {it}")
