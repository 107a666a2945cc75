"""The harness's engine-backed sweep on one small cell (kernel-only timing)."""

import pytest

from frnn_cuda import harness

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_engine_sweep_one_cell():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    res = harness.run_cells([(3, 20000), (12, 20000)], harness.engine_search(), "lowrank", 3, 0.02,
                            log=lambda *a: None)
    for key in ("D3_N20000", "D12_N20000"):
        assert res[key]["latency_ms"] is not None and res[key]["latency_ms"] > 0
        assert res[key]["libfrnn_gpu_ms"] is None
