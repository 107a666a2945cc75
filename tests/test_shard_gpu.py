"""The query-sharded search (frnn_search_sharded) against the whole search.

On one GPU the shard is a one-rank NCCL communicator: every step of the
protocol runs (root plan and build, header and status exchange, broadcast,
slice search, gather, root scatter) and the results must equal
frnn_search_gpu's bit for bit on every path.  With two or more GPUs the same
comparison runs across ranks (tests/shard_worker.py under torchrun), with the
first and the last rank as root."""

import os
import subprocess
import sys

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def one_rank():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    eng = frnn_cuda.FRNNEngine(max_points=400_000)
    shard = frnn_cuda.FRNNShard(eng, 1, 0, frnn_cuda.FRNNShard.unique_id())
    shard.set_timeout(60.0)
    yield frnn_cuda, eng, shard
    shard.close()


def sharded_vs_whole(frnn_cuda, shard, soa, K, r):
    from frnn_cuda.sharded import _DeviceArray
    D, N = soa.shape
    x = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    pi, pd = shard.search(0, x.data_ptr(), N, D, K, r)
    gi = torch.as_tensor(_DeviceArray(pi, (K, N), "<i4"), device="cuda").cpu().numpy()
    gd = torch.as_tensor(_DeviceArray(pd, (K, N), "<f4"), device="cuda").cpu().numpy()
    ref = frnn_cuda.FRNNEngine(max_points=N)
    ref.search_gpu(x.data_ptr(), N, D, K, r)
    ri, rd = ref.get_results_arrays(N, K)
    return gi, gd, ri, rd, ref.last_plan()


@pytest.mark.parametrize("cfg,N", [(1, 60_000), (2, 300_000), (3, 80_000), (4, 60_000), (5, 6_000)])
def test_one_rank_sharded_equals_whole(one_rank, cfg, N):
    frnn_cuda, eng, shard = one_rank
    c = datagen.config(cfg)
    pts, r = datagen.cloud(cfg, N)
    gi, gd, ri, rd, plan = sharded_vs_whole(frnn_cuda, shard, datagen.soa(pts), c.K, r)
    assert_bit_exact(gi, gd, ri, rd, f"cfg{cfg} sharded over one rank, {plan}")
    assert eng.last_plan()["path"] == plan["path"]
    st = shard.last_stats()
    assert st["rows"] == N and st["gather_bytes"] == 0


def test_one_rank_small_brute_force(one_rank):
    frnn_cuda, eng, shard = one_rank
    pts = datagen.generate("uniform", 700, 7, seed=5)
    gi, gd, ri, rd, plan = sharded_vs_whole(frnn_cuda, shard, datagen.soa(pts), 9, 0.3)
    assert plan["path"] == "brute"
    assert_bit_exact(gi, gd, ri, rd, "brute force sharded over one rank")


def test_one_rank_errors_leave_the_shard_usable(one_rank):
    frnn_cuda, eng, shard = one_rank
    with pytest.raises(ValueError):
        shard.search(0, 0, 1000, 3, 8, 0.1)          # the root passes no points
    with pytest.raises(ValueError):
        shard.search(0, 1, 1000, 3, 200, 0.1)        # K > 128
    pts = datagen.generate("uniform", 50_000, 3, seed=6)
    gi, gd, ri, rd, _ = sharded_vs_whole(frnn_cuda, shard, datagen.soa(pts), 8, 0.01)
    assert_bit_exact(gi, gd, ri, rd, "after rejected calls")


def test_stage_times_when_timing_is_on(one_rank):
    frnn_cuda, eng, shard = one_rank
    pts = datagen.generate("mixture", 100_000, 3, seed=8)
    x = torch.from_numpy(datagen.soa(pts)).cuda()
    eng.set_timing(True)
    shard.search(0, x.data_ptr(), 100_000, 3, 16, 0.01)
    st = shard.last_stats()
    eng.set_timing(False)
    assert set(st["stage_ms"]) == set(frnn_cuda.FRNNShard.STAGES)
    assert all(v >= 0 for v in st["stage_ms"].values())


def test_multi_gpu_sharded_equals_whole():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n = min(torch.cuda.device_count(), 4)
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(here, "shard_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert p.returncode == 0 and "SHARD-OK" in p.stdout, p.stdout[-3000:] + p.stderr[-3000:]
