"""Multi-rank host logic of the query-sharded search, on CPU gloo ranks.

Each rank runs ``frnn_cuda.sharded.search_sharded`` with the oracle as its
per-part search (a seeded permutation of the queries stands in for the
engine's cell order, so row ids are not the identity).  The root's assembled
results must equal the oracle's whole-cloud search bit for bit.  Failures are
made on the host: a rank whose part search raises, a rank that exits before
the collectives, a root with a malformed cloud -- every live rank must end with
an error, none may hang."""

import datetime
import multiprocessing as mp
import os
import socket
import sys
import time
import traceback

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cloud(N=3000, D=5, seed=11):
    rng = np.random.default_rng(seed)
    return rng.random((D, N), dtype=np.float64).astype(np.float32)


def _worker(rank, world, port, scenario, q):
    try:
        sys.path[:0] = [os.path.join(ROOT, "pure_cuda-c-_frnn_b200"), os.path.join(ROOT, "oracle")]
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import torch
        import torch.distributed as dist
        import oracle
        from frnn_cuda.sharded import ShardError, search_sharded

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        soa = _cloud()
        D, N = soa.shape
        K, r = 12, 0.22
        perm = np.random.default_rng(5).permutation(N).astype(np.int32)

        def part_search(x, N_, D_, K_, r_, part, nparts):
            if scenario == "raise" and part == 1:
                raise RuntimeError("injected failure")
            if scenario == "die" and part == 1:
                os._exit(3)
            lo, hi = N_ * part // nparts, N_ * (part + 1) // nparts
            ids = perm[lo:hi]
            idx, dst, _ = oracle.search_subset(x.numpy(), ids, K_, r_)
            return torch.from_numpy(ids), torch.from_numpy(idx), torch.from_numpy(dst)

        pts = torch.from_numpy(soa) if rank == 0 else None
        if scenario == "badroot" and rank == 0:
            pts = torch.from_numpy(soa[:, :-1].copy())
        try:
            out = search_sharded(pts, N, D, K, r, part_search)
        except ShardError as exc:
            q.put((rank, "shard_error", str(exc)))
            return
        except Exception as exc:  # a collective broken by a dead peer
            q.put((rank, "error", type(exc).__name__))
            return
        if rank == 0:
            oi, od, _ = oracle.search(soa, K, r)
            ok = np.array_equal(out[0].numpy(), oi) and np.array_equal(out[1].numpy().view(np.int32),
                                                                        od.view(np.int32))
            q.put((rank, "ok" if ok else "mismatch", ""))
        else:
            q.put((rank, "ok" if out is None else "unexpected", ""))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "crash", traceback.format_exc()))


def _run(world, scenario, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    t0 = time.time()
    for p in procs:
        p.join(max(1.0, timeout - (time.time() - t0)))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            raise AssertionError(f"rank {procs.index(p)} hung in scenario {scenario}")
    res = {}
    while not q.empty():
        r, status, msg = q.get()
        res[r] = (status, msg)
    return res, [p.exitcode for p in procs]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_matches_whole_search(world):
    res, codes = _run(world, "ok")
    assert all(res.get(r, ("missing",))[0] == "ok" for r in range(world)), res
    assert codes == [0] * world


def test_failing_part_raises_on_every_rank():
    res, _ = _run(2, "raise")
    assert res[0][0] == "shard_error" and "another rank" in res[0][1], res
    assert res[1][0] == "shard_error" and "injected failure" in res[1][1], res


def test_dead_rank_ends_the_others_with_an_error():
    res, codes = _run(2, "die")
    assert codes[1] == 3
    assert res.get(0, ("missing",))[0] in ("error", "shard_error"), res


def test_malformed_root_cloud_raises_everywhere():
    res, _ = _run(2, "badroot")
    assert res[0][0] == "shard_error" and res[1][0] == "shard_error", res
