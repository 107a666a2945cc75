"""Parity at the benchmark sizes: every configuration at its full N.

The configurations are measured at full size, and full size is where the
paths differ from the small clouds the other files use (a 12M-cell table and
overflowing candidate lists for configuration 2, a 6-axis principal grid of
78M cells for configuration 4, the fp16 filter margin and its overflow pass
for configuration 5).  So each one is searched here at its benchmark size,
through frnn_search_gpu, and checked bit for bit against the CPU oracle:

* configurations 1 and 2: every query (and configuration 2 once more with a
  radius large enough that thousands of candidate lists overflow);
* configurations 3, 4 and 5: a seeded sample of 16,384 queries plus every
  query that went through a fallback pass because its candidate list
  overflowed (frnn_last_overflow).

Against the reference engine itself (compiled from its own sources for
sm_100a): configuration 2 at 1M points (the reference runs its brute force
there), and configurations 3 and 4 at full N (their clouds clipped below 1.0,
because the reference's grid drops points at 1.0, insert_points.cu:74-87).
The bar follows Tests/scripts/validate_correctness.py:108-155 as the project
brief states it: index sets exact except ties at the K-th distance and points
within 1e-6*r^2 of the radius, distances within 1e-5 relative.
"""

import functools
import os

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact, compare_to_reference

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SAMPLE = 16_384


@pytest.fixture(scope="module")
def frnn():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    return frnn_cuda


@functools.lru_cache(maxsize=1)
def full_cloud(cfg):
    c = datagen.config(cfg)
    return datagen.soa(datagen.generate(c.kind, c.N, c.D, seed=datagen.SEED)), c


def engine_search(frnn, soa, K, r):
    D, N = soa.shape
    eng = frnn.FRNNEngine(max_points=N)
    t = torch.from_numpy(soa).cuda()
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    idx, dist = eng.get_results_arrays(N, K)
    plan, overflow = eng.last_plan(), eng.last_overflow()
    del eng, t
    torch.cuda.empty_cache()
    return idx, dist, plan, overflow


EXPECT = {1: ("grid", 3), 2: ("grid", 3), 3: ("grid", 4), 4: ("grid", 6), 5: ("brute_tc", 0)}


@pytest.mark.parametrize("cfg", [1, 2, 3, 4, 5])
def test_full_size_config_vs_oracle(frnn, oracle_mod, cfg):
    soa, c = full_cloud(cfg)
    idx, dist, plan, overflow = engine_search(frnn, soa, c.K, c.radius)
    assert (plan["path"], plan["grid_dims"]) == EXPECT[cfg], plan
    if cfg in (1, 2):
        oi, od, _ = oracle_mod.search(soa, c.K, c.radius)
        assert_bit_exact(idx, dist, oi, od, f"cfg{cfg} full {plan}")
        return
    rng = np.random.default_rng(4321 + cfg)
    sample = rng.choice(c.N, SAMPLE, replace=False).astype(np.int32)
    q = np.union1d(sample, overflow).astype(np.int32)
    oi, od, _ = oracle_mod.search_subset(soa, q, c.K, c.radius)
    assert_bit_exact(idx[:, q], dist[:, q], oi, od,
                     f"cfg{cfg} full, {len(q)} queries ({len(overflow)} overflowed) {plan}")


def test_full_size_overflowing_lists(frnn, oracle_mod):
    """Configuration 2's cloud with a radius 2.2 times its own (about 260
    points in radius on average): many queries overflow the 128-key lists and
    go through the fallback pass; frnn_last_overflow names them, each has more
    than 128 points in radius, and their results are exact."""
    soa, c = full_cloud(2)
    r = 2.2 * c.radius
    idx, dist, plan, overflow = engine_search(frnn, soa, c.K, r)
    assert plan["path"] == "grid" and len(overflow) > 1000, (plan, len(overflow))
    idx128 = oracle_mod.search_subset(soa, overflow[:256].astype(np.int32), 128, r)[0]
    assert (idx128[127] >= 0).all()
    rng = np.random.default_rng(99)
    q = np.union1d(rng.choice(c.N, 4096, replace=False), overflow).astype(np.int32)
    oi, od, _ = oracle_mod.search_subset(soa, q, c.K, r)
    assert_bit_exact(idx[:, q], dist[:, q], oi, od, f"cfg2 x2.2 radius, {len(overflow)} overflowed")


@pytest.fixture(scope="module")
def ref(frnn):
    import oracle
    if not os.path.exists(oracle.REF_SO):
        pytest.skip("reference library not built (make -C oracle ref REF_ROOT=...)")
    return oracle


@pytest.mark.parametrize("cfg", [2, 3, 4])
def test_full_size_config_vs_reference(frnn, ref, cfg):
    soa, c = full_cloud(cfg)
    if cfg in (3, 4):
        # the reference's first-coordinate grid drops points at 1.0
        soa = np.minimum(soa, np.float32(0.999999))
    path = ref.ref_plan(c.N, c.D, c.K, c.radius)["path"]
    assert path == {2: "bf_fallback", 3: "firstd", 4: "firstd"}[cfg], path
    D, N = soa.shape
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    r_eng = ref.RefEngine(N)
    r_eng.search_gpu(t.data_ptr(), N, D, c.K, c.radius)
    ri, rd = r_eng.get_results(N, c.K)
    r_eng.close()
    del t
    ei, ed, _, _ = engine_search(frnn, np.ascontiguousarray(soa), c.K, c.radius)
    st = compare_to_reference(ei, ed, ri, rd, soa, c.radius,
                              d2_f64=lambda qi, pj: ref.pair_d2_f64(soa, qi, pj))
    assert st["mismatch"] == 0 and st["dist_mismatch"] == 0, (cfg, st)
    # nearly every query is identical; the rest are counted ties/boundary cases
    assert st["identical"] >= 0.999 * N, st
