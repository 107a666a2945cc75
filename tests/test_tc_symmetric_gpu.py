"""The symmetric tensor-core filter (FRNN_OPT_TC_SYMMETRIC), through the C ABI.

A whole self-search on the tensor-core path filters each unordered pair of
128-point tiles once and appends every passing pair to both points' candidate
lists; the all-pairs filter (option 0) visits every (query tile, point tile)
pair, as the reference's brute force visits every pair
(frnn/csrc/no_grid_frnn/no_grid_frnn.cu:121-326).  The filter only proposes
candidates and the exact fp32 re-rank decides, so both settings must return
the oracle's arrays bit for bit: odd and even tile counts (the last CTA with
one query block), partial last tiles, lists that overflow into the SIMT
fallback (clusters of identical points), and the diagonal tiles, where a pair
must not be listed twice.
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


def search(frnn, soa, K, r, symmetric):
    D, N = soa.shape
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path("brute_tc")
    eng.set_option(eng.OPT_TC_SYMMETRIC, symmetric)
    t = torch.from_numpy(np.ascontiguousarray(soa, dtype=np.float32)).cuda()
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    assert eng.last_plan()["path"] == "brute_tc"
    idx, dist = eng.get_results_arrays(N, K)
    return idx, dist, eng.last_overflow()


def both_settings(frnn, oracle_mod, soa, K, r, label):
    si, sd, sov = search(frnn, soa, K, r, 1)
    ai, ad, aov = search(frnn, soa, K, r, 0)
    assert_bit_exact(si, sd, ai, ad, f"{label}: symmetric vs all-pairs filter")
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(si, sd, oi, od, f"{label}: symmetric filter vs oracle")
    # both filters list the same pairs, so the same queries overflow
    assert np.array_equal(sov, aov), f"{label}: overflow sets differ"
    return sov


@pytest.mark.parametrize("N", [129, 256, 383, 640, 1000, 2560, 4097])
def test_tile_counts(frnn, oracle_mod, N):
    D = 96
    pts = datagen.generate("sphere", N, D, seed=N)
    r = datagen.calibrate_radius(pts, 24, sample=min(512, N), seed=3)
    both_settings(frnn, oracle_mod, datagen.soa(pts), 32, r, f"N={N}")


@pytest.mark.parametrize("D,K", [(33, 8), (64, 64), (128, 128)])
def test_dims(frnn, oracle_mod, D, K):
    N = 6000
    pts = datagen.generate("sphere", N, D, seed=D + K)
    r = datagen.calibrate_radius(pts, 0.75 * K, sample=512, seed=5)
    both_settings(frnn, oracle_mod, datagen.soa(pts), K, r, f"D={D} K={K}")


def test_overflowing_clusters(frnn, oracle_mod):
    # clusters of identical points larger than a candidate list: their lists
    # fill from both sides of the pairs and overflow to the SIMT fallback
    rng = np.random.default_rng(11)
    D, N = 48, 3000
    centres = rng.standard_normal((6, D)).astype(np.float32)
    pts = rng.standard_normal((N, D)).astype(np.float32)
    pts[:1800] = centres[np.arange(1800) % 6]
    r = 0.5
    ov = both_settings(frnn, oracle_mod, datagen.soa(pts), 16, r, "clusters")
    assert len(ov) >= 1800, len(ov)
