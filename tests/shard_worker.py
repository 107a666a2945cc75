"""One rank of the multi-GPU sharded-search test (run under torchrun by
tests/test_shard_gpu.py; not collected by pytest itself).

Every rank joins an FRNNShard; for each case the root's cloud is searched
sharded (root 0, then the last rank as root) and the root compares the
gathered [K, N] results bit for bit with a whole search on its own GPU."""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "pure_cuda-c-_frnn_b200"), os.path.join(ROOT, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import datetime  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import frnn_cuda  # noqa: E402
from frnn_cuda import datagen  # noqa: E402
from frnn_cuda.sharded import _DeviceArray, nccl_shard  # noqa: E402
from parity import assert_bit_exact  # noqa: E402

CASES = [(1, 60_000), (2, 200_000), (3, 60_000), (4, 60_000), (5, 9_000)]


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    eng = frnn_cuda.FRNNEngine(max_points=200_000, device=local)
    shard = nccl_shard(eng)
    shard.set_timeout(60.0)
    ref = frnn_cuda.FRNNEngine(max_points=200_000, device=local)
    for cfg, N in CASES:
        c = datagen.config(cfg)
        pts, r = datagen.cloud(cfg, N)
        soa = datagen.soa(pts)
        x = torch.from_numpy(soa).cuda()
        for root in (0, world - 1):
            pi, pd = shard.search(root, x.data_ptr() if rank == root else 0, N, c.D, c.K, r)
            st = shard.last_stats()
            if rank == root:
                # copy out of the shard's buffers (valid until its next call)
                got_i = torch.as_tensor(_DeviceArray(pi, (c.K, N), "<i4"), device="cuda").cpu()
                got_d = torch.as_tensor(_DeviceArray(pd, (c.K, N), "<f4"), device="cuda").cpu()
                ref.search_gpu(x.data_ptr(), N, c.D, c.K, r)
                ri, rd = ref.get_results_arrays(N, c.K)
                assert_bit_exact(got_i.cpu().numpy(), got_d.cpu().numpy(), ri, rd,
                                 f"cfg{cfg} N={N} root={root} world={world} {eng.last_plan()}")
                print(f"rank {rank} cfg{cfg} root={root} ok {eng.last_plan()} {st}", flush=True)
            else:
                assert pi == 0 and pd == 0
            assert st["rows"] >= 0
        dist.barrier()
    # the tensor-core path with the symmetric filter shared between the ranks
    # (each rank appends into the others' lists) and without it, on a cloud
    # whose last tile is partial and on one whose lists overflow
    rng = np.random.default_rng(5)
    clusters = rng.standard_normal((3000, 48)).astype(np.float32)
    clusters[:1800] = clusters[np.arange(1800) % 6]
    tc_cases = [("sphere", datagen.soa(datagen.generate("sphere", 9001, 128, seed=9)), 128, None),
                ("clusters", datagen.soa(clusters), 16, 0.5)]
    for name, soa, K, r in tc_cases:
        D, N = soa.shape
        if r is None:
            r = datagen.calibrate_radius(np.ascontiguousarray(soa.T), 64, sample=512)
        x = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
        for sym in (1, 0):
            shard.set_option(shard.OPT_TC_SYMMETRIC, sym)
            pi, pd = shard.search(0, x.data_ptr() if rank == 0 else 0, N, D, K, r)
            if rank == 0:
                got_i = torch.as_tensor(_DeviceArray(pi, (K, N), "<i4"), device="cuda").cpu()
                got_d = torch.as_tensor(_DeviceArray(pd, (K, N), "<f4"), device="cuda").cpu()
                ref.set_path("brute_tc")
                ref.search_gpu(x.data_ptr(), N, D, K, r)
                ref.set_path("auto")
                ri, rd = ref.get_results_arrays(N, K)
                assert_bit_exact(got_i.numpy(), got_d.numpy(), ri, rd, f"tc {name} sym={sym} world={world}")
                print(f"rank {rank} tc {name} sym={sym} ok {eng.last_plan()} {shard.last_stats()}", flush=True)
        shard.set_option(shard.OPT_TC_SYMMETRIC, 1)
        dist.barrier()
    shard.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("SHARD-OK", flush=True)


if __name__ == "__main__":
    main()
