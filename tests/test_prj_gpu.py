"""The principal-axis search kernel (grid_prj.cuh) under stress, against the oracle.

The kernel queues (candidate, query) pairs that pass the projected screen and
finishes them 32 at a time; a list near its capacity is compacted to its K
smallest keys.  These clouds push every part of that: dense clusters of
duplicated points (whole chunks of 32 candidates passing for all 8 queries of
a group, so a chunk adds 256 pairs to the queue; exact distance ties broken by
index), small K against many neighbours (a compaction on almost every pass),
K = 128 (the largest lists), and K above the neighbour count (padding rows).
The list search is switched off so K <= 32 also runs this kernel."""

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


def clustered_cloud(D: int, n_base: int, n_sites: int, copies: int, seed: int) -> np.ndarray:
    """A rank-6 cloud plus `copies` exact copies of each of `n_sites` of its
    points, shuffled."""
    rng = np.random.default_rng(seed)
    base = np.minimum(datagen.generate("lowrank6", n_base, D, seed=seed), np.float32(0.999999))
    sites = base[rng.choice(n_base, n_sites, replace=False)]
    pts = np.concatenate([base, np.repeat(sites, copies, axis=0)])
    return pts[rng.permutation(len(pts))].astype(np.float32)


def search(frnn, soa, K, r):
    D, N = soa.shape
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path("grid")
    eng.set_option(eng.OPT_GRID_AXES, eng.GRID_AXES_PRINCIPAL)
    eng.set_option(eng.OPT_LIST_SEARCH, eng.LIST_SEARCH_NEVER)
    x = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    i, d = eng.get_results_arrays(N, K)
    return i, d, eng.last_plan()


@pytest.mark.parametrize("K", [1, 8, 64, 128])
@pytest.mark.parametrize("D", [8, 16])
def test_duplicate_clusters(frnn, oracle_mod, D, K):
    pts = clustered_cloud(D, 20_000, 40, 60, seed=11 + D)
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(pts, 40.0, sample=512)
    i, d, plan = search(frnn, soa, K, r)
    assert plan["path"] == "grid" and plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, f"clusters D={D} K={K} {plan}")


@pytest.mark.parametrize("K", [4, 33])
def test_many_neighbours_small_lists(frnn, oracle_mod, K):
    # about 300 neighbours per query: lists are compacted again and again
    pts = np.minimum(datagen.generate("lowrank6", 30_000, 16, seed=5), np.float32(0.999999))
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(pts, 300.0, sample=512)
    i, d, plan = search(frnn, soa, K, r)
    assert plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(i, d, oi, od, f"dense K={K}")


def test_k_above_neighbour_count(frnn, oracle_mod):
    pts = np.minimum(datagen.generate("lowrank4", 25_000, 12, seed=6), np.float32(0.999999))
    soa = datagen.soa(pts)
    r = datagen.calibrate_radius(pts, 6.0, sample=512)
    i, d, plan = search(frnn, soa, 128, r)
    assert plan["axes"] == "principal", plan
    oi, od, _ = oracle_mod.search(soa, 128, r)
    assert_bit_exact(i, d, oi, od, "sparse K=128")
    assert (i[-1] == -1).all()  # padding rows past every query's neighbours
