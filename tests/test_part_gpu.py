"""frnn_search_gpu_part on the GPU: the parts of a search, put back together by
their row ids, must equal the whole search bit for bit and cover every query
once -- on every path (D = 3 collect/emit, D = 3 cooperative, ND grid, SIMT
brute force, tensor-core brute force).  The sharded driver is also run on one
NCCL rank with the engine as its part search."""

import datetime
import os
import socket

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


def whole(frnn, x, N, D, K, r, path):
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path(path)
    eng.search_gpu(x.data_ptr(), N, D, K, r)
    i, d = eng.get_results_arrays(N, K)
    return i, d, eng.last_plan()["path"]


def assembled(frnn, x, N, D, K, r, path, nparts):
    from frnn_cuda.sharded import engine_part_search
    eng = frnn.FRNNEngine(max_points=N)
    eng.set_path(path)
    run = engine_part_search(eng)
    idx = np.full((K, N), -7, np.int32)
    dst = np.zeros((K, N), np.float32)
    seen = np.zeros(N, np.int64)
    for p in range(nparts):
        ids, i, d = run(x, N, D, K, r, p, nparts)
        ids = ids.cpu().numpy()
        idx[:, ids] = i.cpu().numpy()
        dst[:, ids] = d.cpu().numpy()
        np.add.at(seen, ids, 1)
    assert (seen == 1).all(), "parts must cover every query once"
    return idx, dst


CASES = [
    ("uniform", 3, 20000, 16, "grid"),      # D = 3 collect / emit
    ("mixture", 3, 20000, 48, "grid"),      # D = 3 cooperative kernel
    ("lowrank4", 7, 12000, 20, "grid"),     # grid on 4 axes, full-D ranking
    ("uniform", 5, 3000, 8, "brute"),       # SIMT brute force
    ("sphere", 64, 5000, 32, "brute_tc"),   # tensor-core filter
]


@pytest.mark.parametrize("kind,D,N,K,path", CASES)
@pytest.mark.parametrize("nparts", [1, 2, 3, 7])
def test_parts_equal_whole(frnn, kind, D, N, K, path, nparts):
    pts = datagen.generate(kind, N, D, seed=D + N)
    soa = datagen.soa(pts)
    sample = np.ascontiguousarray(soa.T)
    r = datagen.calibrate_radius(sample, 24, sample=512, seed=3)
    x = torch.from_numpy(soa).cuda()
    wi, wd, wpath = whole(frnn, x, N, D, K, r, path)
    assert wpath == path
    pi, pd = assembled(frnn, x, N, D, K, r, path, nparts)
    assert_bit_exact(pi, pd, wi, wd, f"{kind} D={D} {path} parts={nparts}")


def test_more_parts_than_tiles(frnn):
    # tensor-core parts are whole 128-query tiles: some parts are empty
    N, D, K = 300, 40, 8
    soa = datagen.soa(datagen.generate("sphere", N, D, seed=1))
    x = torch.from_numpy(soa).cuda()
    wi, wd, _ = whole(frnn, x, N, D, K, 1.2, "brute_tc")
    pi, pd = assembled(frnn, x, N, D, K, 1.2, "brute_tc", 5)
    assert_bit_exact(pi, pd, wi, wd, "empty parts")


def test_part_arguments_rejected(frnn):
    eng = frnn.FRNNEngine(max_points=100)
    x = torch.rand(3, 100, device="cuda")
    with pytest.raises(ValueError):
        eng.search_gpu_part(x.data_ptr(), 100, 3, 4, 0.1, 2, 2)
    with pytest.raises(ValueError):
        eng.search_gpu_part(x.data_ptr(), 100, 3, 4, 0.1, 0, 0)


def test_sharded_driver_one_nccl_rank(frnn):
    import torch.distributed as dist
    from frnn_cuda.sharded import engine_part_search, search_sharded
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        c = datagen.config(1)
        pts, r = datagen.cloud(1, 30000)
        soa = datagen.soa(pts)
        x = torch.from_numpy(soa).cuda()
        eng = frnn.FRNNEngine(max_points=30000)
        oi, od = search_sharded(x, 30000, 3, c.K, r, engine_part_search(eng))
        wi, wd, _ = whole(frnn, x, 30000, 3, c.K, r, "grid")
        assert_bit_exact(oi.cpu().numpy(), od.cpu().numpy(), wi, wd, "sharded x1")
    finally:
        dist.destroy_process_group()
