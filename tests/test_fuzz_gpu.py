"""Seeded random cases across the whole input space, checked bit for bit
against the oracle.

Each case draws a distribution, a dimension, a size, K, a radius (a quantile of
the cloud's own neighbour distances, so the in-radius counts range from none
to well past K), a path and an entry point from a fixed seed, so a failure
reproduces by its case number.  The structured tests pin each feature; this
file looks for interactions between them (ragged tiles, lists that overflow,
empty cells, edge clamping, separate query sets, built grids)."""

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

N_CASES = 48


@pytest.fixture(scope="module")
def frnn():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    return frnn_cuda


def draw(case):
    """The case's parameters: (points, queries or None, K, r, path, entry)."""
    rng = np.random.default_rng(1000 + case)
    kind = rng.choice(["uniform", "mixture", "lowrank4", "lowrank6", "sphere", "dups"])
    if kind == "sphere":
        D = int(rng.choice([3, 8, 33, 64, 100, 128]))
    elif kind in ("lowrank4", "lowrank6"):
        D = int(rng.choice([7, 9, 12, 16, 20, 32]))
    else:
        D = int(rng.choice([1, 2, 3, 3, 3, 4, 5, 6]))
    N = int(rng.choice([1, 2, 37, 128, 129, 1000, 4097, 12000, 30000]))
    K = int(rng.choice([1, 2, 7, 16, 17, 32, 33, 64, 100, 128]))
    if kind == "dups":
        base = rng.random((max(1, N // 20), D)).astype(np.float32)
        pts = base[rng.integers(0, len(base), N)]
    else:
        pts = datagen.generate(kind, N, D, seed=case)
    # radius: a quantile of the distance to a random point's k-th neighbour
    m = min(N, 256)
    sample = pts[rng.choice(N, m, replace=False)]
    d2 = ((sample[:, None, :].astype(np.float64) - pts[None, :, :]) ** 2).sum(-1)
    kth = int(rng.choice([1, 4, 16, 64, 256]))
    dk = np.sort(d2, axis=1)[:, min(kth, N - 1)]
    r = float(np.sqrt(np.quantile(dk, rng.choice([0.1, 0.5, 0.9])))) or 1e-3
    if D > 32:
        path = str(rng.choice(["auto", "brute", "brute_tc"]))
    else:
        path = str(rng.choice(["auto", "auto", "grid", "brute"]))
    entry = str(rng.choice(["points", "points", "queries", "built"]))
    if entry != "points" and N < 2:
        entry = "points"
    q = None
    if entry != "points":
        M = int(rng.choice([1, 50, 777, 5000]))
        lo, hi = pts.min(0), pts.max(0)
        q = (lo - 0.1 * (hi - lo) + rng.random((M, D)) * 1.2 * (hi - lo)).astype(np.float32)
        q[: M // 3] = pts[rng.integers(0, N, M // 3)]
    if entry == "built" and path == "brute":
        path = "auto"
    return pts, q, K, r, path, entry


@pytest.mark.parametrize("case", range(N_CASES))
def test_random_case(frnn, oracle_mod, case):
    pts, q, K, r, path, entry = draw(case)
    N, D = pts.shape
    eng = frnn.FRNNEngine(max_points=N)
    if path != "auto":
        eng.set_path(path)
    xp = torch.from_numpy(datagen.soa(pts)).cuda()
    what = f"case {case}: N={N} D={D} K={K} r={r:.4g} path={path} entry={entry}"
    if entry == "points":
        eng.search_gpu(xp.data_ptr(), N, D, K, r)
        i, d = eng.get_results_arrays(N, K)
        oi, od, _ = oracle_mod.search(datagen.soa(pts), K, r)
    else:
        M = q.shape[0]
        xq = torch.from_numpy(datagen.soa(q)).cuda()
        if entry == "queries":
            eng.search_gpu_queries(xp.data_ptr(), N, xq.data_ptr(), M, D, K, r)
        else:
            eng.build_grid(xp.data_ptr(), N, D, r)
            eng.query_grid(xq.data_ptr(), M, K)
        i, d = eng.get_results_arrays(M, K)
        oi, od, _ = oracle_mod.search_queries(datagen.soa(pts), datagen.soa(q), K, r)
    assert_bit_exact(i, d, oi, od, what + f" plan={eng.last_plan()}")
