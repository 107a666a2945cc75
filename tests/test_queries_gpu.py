"""frnn_search_gpu_queries: a separate query set against a point set.

Every path is forced in turn and compared bit for bit with the oracle's exact
search of the same queries (oracle_search_queries).  The queries mix points
inside the cloud, points outside its bounding box (within r of it and far
away) and exact copies of cloud points (distance 0)."""

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


def queries_for(pts, M, r, seed):
    """M queries: a third jittered cloud points, a third copies of cloud
    points, the rest spread over a box 10 % larger than the cloud's (some of
    them within r outside it) plus a few far away."""
    rng = np.random.default_rng(seed)
    N, D = pts.shape
    lo, hi = pts.min(0), pts.max(0)
    a = M // 3
    q1 = pts[rng.integers(0, N, a)] + rng.normal(0, r, (a, D))
    q2 = pts[rng.integers(0, N, a)]
    q3 = lo - 0.05 * (hi - lo) + rng.random((M - 2 * a, D)) * 1.1 * (hi - lo)
    q3[:5] += 100.0 * (hi - lo + 1.0)
    q = np.concatenate([q1, q2, q3]).astype(np.float32)
    return q[rng.permutation(M)]


def run(frnn, pts, q, K, r, path, axes=None):
    N, D = pts.shape
    M = q.shape[0]
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path(path)
    if axes is not None:
        eng.set_option(eng.OPT_GRID_AXES, axes)
    xp = torch.from_numpy(datagen.soa(pts)).cuda()
    xq = torch.from_numpy(datagen.soa(q)).cuda()
    eng.search_gpu_queries(xp.data_ptr(), N, xq.data_ptr(), M, D, K, r)
    i, d = eng.get_results_arrays(M, K)
    return i, d, eng.last_plan()


CASES = [
    # kind, D, N, M, K, path, axes
    ("uniform", 3, 30000, 20000, 16, "grid", None),      # D = 3 collect / emit
    ("mixture", 3, 30000, 45000, 48, "grid", None),      # D = 3 cooperative
    ("uniform", 2, 20000, 7000, 8, "grid", None),        # full-D grid, G = 2
    ("lowrank4", 7, 20000, 9000, 20, "grid", 1),         # leading coordinates
    ("lowrank6", 16, 20000, 9000, 20, "grid", 2),        # principal axes
    ("uniform", 5, 3000, 2500, 8, "brute", None),        # SIMT brute force
    ("sphere", 64, 6000, 3000, 32, "brute_tc", None),    # tensor-core filter
    ("sphere", 128, 3000, 5000, 128, "brute_tc", None),
]


@pytest.mark.parametrize("kind,D,N,M,K,path,axes", CASES)
def test_query_set_matches_oracle(frnn, oracle_mod, kind, D, N, M, K, path, axes):
    pts = datagen.generate(kind, N, D, seed=N + D)
    r = datagen.calibrate_radius(pts, 20, sample=512, seed=3)
    q = queries_for(pts, M, r, seed=D)
    i, d, plan = run(frnn, pts, q, K, r, path, axes)
    assert plan["path"] == path, plan
    if axes == 2:
        assert plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search_queries(datagen.soa(pts), datagen.soa(q), K, r)
    assert_bit_exact(i, d, oi, od, f"{kind} D={D} {plan}")


def test_query_set_equal_to_points_is_the_self_search(frnn):
    N, D, K = 20000, 3, 16
    pts = datagen.generate("uniform", N, D, seed=5)
    r = datagen.uniform_radius(N, D, 16)
    eng = frnn.FRNNEngine(max_points=N)
    x = torch.from_numpy(datagen.soa(pts)).cuda()
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    a = eng.get_results_arrays(N, K)
    eng.search_gpu_queries(x.data_ptr(), N, x.data_ptr(), N, D, K, r)
    b = eng.get_results_arrays(N, K)
    assert_bit_exact(a[0], a[1], b[0], b[1], "queries == points")


def test_query_set_rejects_bad_arguments(frnn):
    eng = frnn.FRNNEngine(max_points=100)
    x = torch.rand(3, 100, device="cuda")
    q = torch.rand(3, 10, device="cuda")
    with pytest.raises(ValueError):
        eng.search_gpu_queries(x.data_ptr(), 100, q.data_ptr(), 0, 3, 4, 0.1)
    with pytest.raises(ValueError):
        eng.search_gpu_queries(x.data_ptr(), 100, 0, 10, 3, 4, 0.1)
    qn = q.clone()
    qn[0, 3] = float("nan")
    eng.set_path("grid")
    pts = torch.rand(3, 100, device="cuda")
    with pytest.raises(ValueError):
        eng.search_gpu_queries(pts.data_ptr(), 100, qn.data_ptr(), 10, 3, 4, 0.2)


@pytest.mark.parametrize("kind,D,N,path", [("uniform", 3, 30000, "grid"), ("lowrank6", 16, 20000, "grid"),
                                           ("mixture", 5, 20000, "grid"), ("sphere", 64, 5000, "brute_tc")])
def test_build_once_query_many(frnn, oracle_mod, kind, D, N, path):
    pts = datagen.generate(kind, N, D, seed=N + 2 * D)
    r = datagen.calibrate_radius(pts, 20, sample=512, seed=4)
    eng = frnn.FRNNEngine(max_points=N)
    xp = torch.from_numpy(datagen.soa(pts)).cuda()
    eng.build_grid(xp.data_ptr(), N, D, r)
    for t, (M, K) in enumerate([(7000, 16), (2500, 40), (9000, 1)]):
        q = queries_for(pts, M, r, seed=10 * D + t)
        xq = torch.from_numpy(datagen.soa(q)).cuda()
        eng.query_grid(xq.data_ptr(), M, K)
        i, d = eng.get_results_arrays(M, K)
        assert eng.last_plan()["path"] == path
        oi, od, _ = oracle_mod.search_queries(datagen.soa(pts), datagen.soa(q), K, r)
        assert_bit_exact(i, d, oi, od, f"{kind} D={D} M={M} K={K}")


def test_other_search_discards_the_built_grid(frnn):
    N, D = 20000, 3
    pts = torch.rand(D, N, device="cuda")
    q = torch.rand(D, 100, device="cuda")
    eng = frnn.FRNNEngine(max_points=N)
    with pytest.raises(frnn.FRNNError):
        eng.query_grid(q.data_ptr(), 100, 4)
    eng.build_grid(pts.data_ptr(), N, D, 0.02)
    eng.query_grid(q.data_ptr(), 100, 4)
    eng.search_gpu(pts.data_ptr(), N, D, 4, 0.02)
    with pytest.raises(frnn.FRNNError):
        eng.query_grid(q.data_ptr(), 100, 4)
