"""The sharded symmetric tensor-core filter's protocol, on CPU gloo ranks.

The GPU code (csrc/shard.cu: tc_sym_setup, tc_sym_range; bf_tc.cu:
filter_kernel with sym, tc_pull_kernel) is checked on B200s by
test_shard_gpu.py and shard_worker.py.  This file restates the protocol with
numpy on gloo ranks, so the rules it rests on are pinned without a GPU:

* ranks own the queries frnn_shard_tc_partition gives them (the engine's own
  host function), in whole pairs of 128-query blocks;
* rank r filters each of its blocks b against the point tiles t >= b, keeping
  every passing pair in its own lists: q gets p always, p gets q only off the
  diagonal tile (on it, the transposed element lists the pair);
* after a barrier every rank pulls, for each of its own queries, the entries
  the other ranks listed for it.

Each query's merged list must be exactly its in-radius set, every pair
listed once, and every query owned by exactly one rank.  (The reference's
brute force visits every ordered pair on one GPU, no_grid_frnn.cu:121-326.)
"""

import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TILE = 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, N, q):
    try:
        sys.path[:0] = [os.path.join(ROOT, "pure_cuda-c-_frnn_b200")]
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import torch
        import torch.distributed as dist
        import frnn_cuda

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        # the root's cloud, broadcast to every rank
        pts = torch.zeros((N, 6), dtype=torch.float64)
        if rank == 0:
            pts = torch.from_numpy(np.random.default_rng(3).random((N, 6)))
        dist.broadcast(pts, 0)
        x = pts.numpy()
        r2 = 0.35 ** 2
        bounds = frnn_cuda.shard_tc_partition(N, world)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        T = (N + TILE - 1) // TILE

        # this rank's share of the triangle: its blocks against tiles t >= b
        lists = [[] for _ in range(N)]
        for b in range(lo // TILE, (hi + TILE - 1) // TILE):
            qs = np.arange(b * TILE, min(N, (b + 1) * TILE))
            for t in range(b, T):
                ps = np.arange(t * TILE, min(N, (t + 1) * TILE))
                d2 = ((x[qs][:, None, :] - x[ps][None, :, :]) ** 2).sum(-1)
                for i, j in zip(*np.nonzero(d2 < r2)):
                    lists[qs[i]].append(int(ps[j]))
                    if t != b:
                        lists[ps[j]].append(int(qs[i]))
        dist.barrier()  # every rank's filter has finished
        # the pull: each rank's entries for this rank's queries
        every = [None] * world
        dist.all_gather_object(every, lists)
        bad = []
        for qi in range(lo, hi):
            merged = [p for src in every for p in src[qi]]
            truth = np.nonzero(((x - x[qi]) ** 2).sum(-1) < r2)[0].tolist()
            if len(merged) != len(set(merged)) or sorted(merged) != truth:
                bad.append(qi)
        owned = torch.tensor([hi - lo], dtype=torch.int64)
        dist.all_reduce(owned)
        q.put((rank, "ok" if not bad and int(owned) == N and lo % (2 * TILE) == 0 else f"bad {bad[:5]}",
               (lo, hi, int(owned))))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,N", [(2, 2000), (3, 1500)])
def test_symmetric_shares_and_pull_list_every_pair_once(world, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, info in sorted(results):
        assert status == "ok", (rank, status, info)
