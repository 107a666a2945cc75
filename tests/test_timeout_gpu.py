"""The bounded device waits give up, report FRNN_ERR_TIMEOUT, and leave the
engine usable.

Two waits spin on progress made by other threads: the prefix scan's
look-back (a tile waits for its predecessors' published sums) and the
tensor-core filter's mbarrier waits (the MMA thread waits for the producer's
copies).  FRNN_OPT_TEST_STALL makes each run out on purpose -- a scan tile
that never publishes its status, a point tile the producer never copies --
so nothing faults: the waiting side gives up after its limit, sets the error
flag and returns, the host reports FRNN_ERR_TIMEOUT, and the next search on
the same engine is bit-exact with the oracle.  (The reference checks no such
condition; its only error report is one print, no_grid_frnn.cu:321-324.)
"""

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TIMEOUT = 4


@pytest.fixture(scope="module")
def frnn():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    return frnn_cuda


def stalled_then_clean(frnn, oracle_mod, soa, K, r, stall, want_path):
    D, N = soa.shape
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_option(eng.OPT_TEST_STALL, stall)
    with pytest.raises(frnn.FRNNError) as err:
        eng.search_gpu(t.data_ptr(), N, D, K, r)
    assert err.value.status == TIMEOUT, err.value
    assert "gave up" in str(err.value)
    # the same engine, the knob off: a normal, exact search
    eng.set_option(eng.OPT_TEST_STALL, eng.TEST_STALL_OFF)
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    assert eng.last_plan()["path"] == want_path
    idx, dist = eng.get_results_arrays(N, K)
    oi, od, _ = oracle_mod.search(soa, K, r)
    assert_bit_exact(idx, dist, oi, od, f"after a {want_path} timeout")
    # and once more, to show no state of the stalled search is left over
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    idx2, dist2 = eng.get_results_arrays(N, K)
    assert_bit_exact(idx2, dist2, oi, od, "second search after the timeout")


def test_scan_lookback_gives_up(frnn, oracle_mod):
    pts, r = datagen.cloud(1, 60_000)          # ~16K cells: four scan tiles
    stalled_then_clean(frnn, oracle_mod, datagen.soa(pts), 16, r, 1, "grid")


def test_scan_lookback_gives_up_principal_grid(frnn, oracle_mod):
    pts, r = datagen.cloud(3, 40_000)
    stalled_then_clean(frnn, oracle_mod, datagen.soa(pts), 32, r, 1, "grid")


def test_tc_filter_wait_gives_up(frnn, oracle_mod):
    pts, r = datagen.cloud(5, 2_000)           # 16 point tiles; tile 1 never arrives
    stalled_then_clean(frnn, oracle_mod, datagen.soa(pts), 16, r, 2, "brute_tc")


def test_stall_option_is_validated(frnn):
    eng = frnn.FRNNEngine(max_points=16)
    with pytest.raises(ValueError):
        eng.set_option(eng.OPT_TEST_STALL, 3)
