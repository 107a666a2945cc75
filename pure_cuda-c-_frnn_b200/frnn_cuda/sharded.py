"""Query-sharded search of one cloud over the ranks of a torch.distributed group.

Two forms of the same protocol:

* ``nccl_shard(engine)`` -- the engine's own NCCL path (frnn_search_sharded in
  the C ABI, csrc/shard.cu): the root builds the search structure once and
  broadcasts it, every rank searches a slice of the cell-sorted queries of
  equal estimated work, and one kernel on the root scatters the gathered
  slices.  torch.distributed only carries the 128-byte NCCL id at set-up;
  no tensor of the search passes through torch.
* ``search_sharded(points, ..., part_search)`` -- the same steps written with
  torch.distributed collectives around a ``part_search`` callable, so that the
  protocol (including its failure handling) runs on CPU ranks over gloo with
  the oracle as the part search.

The reference searches a cloud on one GPU (``FRNNEngine.search_gpu``,
python_interface/frnn_engine.cu:195-250).  Queries are independent and the
point set is read-only, so a cloud splits over ranks (one process per GPU) by
query:

  1. the root's cloud (SoA, ``[D, N]`` float32) is broadcast to every rank;
  2. every rank runs ``part_search`` for its part ``rank`` of ``world`` -- with
     the CUDA engine, ``FRNNEngine.search_gpu_part``: each rank builds the same
     grid and searches one contiguous slice of the cell-sorted queries, so
     neighbouring queries share cache lines on one GPU;
  3. every rank reports success or failure in one all-reduce, so a rank whose
     search failed makes every rank raise ``ShardError`` instead of leaving the
     others waiting in the gather;
  4. the slices (row ids, K x rows indices and distances) are gathered to the
     root, which scatters them into the ``[K, N]`` result arrays.

The results are identical to a single engine's ``search_gpu`` on the whole
cloud.  The collectives are the group's own (NCCL between GPUs, gloo on CPU),
so the same code runs the CPU tests with the oracle as ``part_search``.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["ShardError", "engine_part_search", "nccl_shard", "search_sharded"]


class ShardError(RuntimeError):
    """A rank's part of a sharded search failed; raised on every rank."""


class _DeviceArray:
    """Zero-copy view of an engine-owned device array (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def nccl_shard(engine, group=None, src: int = 0):
    """This rank's ``FRNNShard`` for ``engine``: rank ``src`` of ``group``
    makes the NCCL id and every rank receives it (a host-side broadcast over
    the group); collective."""
    from frnn_cuda import FRNNShard
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    src_global = dist.get_global_rank(group, src) if group is not None else src
    box = [FRNNShard.unique_id() if rank == src else None]
    dist.broadcast_object_list(box, src=src_global, group=group)
    return FRNNShard(engine, world, rank, box[0])


def engine_part_search(engine) -> Callable:
    """``part_search`` backed by a CUDA ``FRNNEngine`` (the results are copied
    out of the engine's buffers, which the next call reuses)."""

    def run(x: torch.Tensor, N: int, D: int, K: int, radius: float, part: int, nparts: int):
        n, pr, pi, pd = engine.search_gpu_part(x.data_ptr(), N, D, K, radius, part, nparts)
        if n == 0:
            e = torch.empty(0, dtype=torch.int32, device=x.device)
            return e, torch.empty((K, 0), dtype=torch.int32, device=x.device), \
                torch.empty((K, 0), dtype=torch.float32, device=x.device)
        ids = torch.as_tensor(_DeviceArray(pr, (n,), "<i4"), device=x.device).clone()
        idx = torch.as_tensor(_DeviceArray(pi, (K, n), "<i4"), device=x.device).clone()
        dst = torch.as_tensor(_DeviceArray(pd, (K, n), "<f4"), device=x.device).clone()
        return ids, idx, dst

    return run


def search_sharded(points: Optional[torch.Tensor], N: int, D: int, K: int, radius: float,
                   part_search: Callable, group=None, root: int = 0,
                   device: Optional[torch.device] = None):
    """Search the root's cloud with every rank of ``group`` taking one part.

    ``points`` is the root's ``[D, N]`` float32 SoA tensor (ignored elsewhere);
    ``part_search(x, N, D, K, radius, part, nparts)`` returns
    ``(row_ids [n], idx [K, n], dist [K, n])`` for one part.  ``root`` is a
    rank of ``group``.  Returns ``(idx [K, N] int32, dist [K, N] float32)`` on
    the root and ``None`` on the other ranks.  Every rank makes the same
    collective calls in the same order, on the error path too.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    root_global = dist.get_global_rank(group, root) if group is not None else root
    if device is None:
        device = points.device if (rank == root and points is not None) else (
            torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
            else torch.device("cpu"))

    # 1. the cloud
    if rank == root:
        if points is None or tuple(points.shape) != (D, N) or points.dtype != torch.float32:
            x = torch.empty((D, N), dtype=torch.float32, device=device)
            bad = 1
        else:
            x = points.to(device).contiguous()
            bad = 0
    else:
        x = torch.empty((D, N), dtype=torch.float32, device=device)
        bad = 0
    flag = torch.tensor([bad], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    if int(flag.item()):
        raise ShardError(f"the root's points must be a float32 tensor of shape ({D}, {N})")
    dist.broadcast(x, src=root_global, group=group)

    # 2. this rank's part
    err = None
    try:
        ids, idx, dst = part_search(x, N, D, K, radius, rank, world)
        ids = ids.to(device=device, dtype=torch.int32).contiguous()
        idx = idx.to(device=device, dtype=torch.int32).reshape(K, -1).contiguous()
        dst = dst.to(device=device, dtype=torch.float32).reshape(K, -1).contiguous()
        n = ids.numel()
        if idx.shape[1] != n or dst.shape[1] != n:
            raise ValueError("row ids and result columns differ in length")
    except Exception as exc:  # reported to every rank below
        err = exc
        n = 0

    # 3. every rank learns whether any part failed, and the largest slice
    stat = torch.tensor([1 if err is not None else 0, n], dtype=torch.int64, device=device)
    dist.all_reduce(stat, op=dist.ReduceOp.MAX, group=group)
    if int(stat[0].item()):
        if err is not None:
            raise ShardError(f"rank {rank}: part search failed: {err}") from err
        raise ShardError("another rank's part search failed")
    nmax = int(stat[1].item())

    # 4. gather the padded slices to the root
    pad_ids = torch.full((nmax,), -1, dtype=torch.int32, device=device)
    pad_idx = torch.empty((K, nmax), dtype=torch.int32, device=device)
    pad_dst = torch.empty((K, nmax), dtype=torch.float32, device=device)
    pad_ids[:n] = ids
    pad_idx[:, :n] = idx
    pad_dst[:, :n] = dst
    outs = []
    for t in (pad_ids, pad_idx, pad_dst):
        glist = [torch.empty_like(t) for _ in range(world)] if rank == root else None
        dist.gather(t, gather_list=glist, dst=root_global, group=group)
        outs.append(glist)
    if rank != root:
        return None
    out_idx = torch.empty((K, N), dtype=torch.int32, device=device)
    out_dst = torch.empty((K, N), dtype=torch.float32, device=device)
    seen = torch.zeros(N, dtype=torch.int32, device=device)
    for r_ids, r_idx, r_dst in zip(*outs):
        keep = r_ids >= 0
        cols = r_ids[keep].long()
        out_idx[:, cols] = r_idx[:, keep]
        out_dst[:, cols] = r_dst[:, keep]
        seen.index_add_(0, cols, torch.ones_like(cols, dtype=torch.int32))
    if not bool((seen == 1).all()):
        raise ShardError("the parts do not cover every query exactly once")
    return out_idx, out_dst
