"""frnn_cuda -- B200 fixed-radius nearest-neighbour engine.

Drop-in for the reference's Python module of the same name
(python_interface/nanobind_module.cu:8-21 in DebuRatnam/Pure_CUDA-C-_FRNN):

    engine = frnn_cuda.FRNNEngine(max_points=N)
    idxs, dists = engine.search(points, K, radius)          # host AoS in, lists out
    idx_ptr, dist_ptr = engine.search_gpu(dev_ptr, N, dim, K, radius)
    idxs, dists = engine.get_results(N, K)                  # SoA lists

The module is a ctypes binding of the C ABI in include/frnn_b200.h, which is
implemented by libfrnn_b200.so (hand-written sm_100a CUDA kernels).  There is
no fallback: if the library or a B200-class device is missing, constructing an
engine raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Sequence

import numpy as np

__all__ = ["FRNNEngine", "FRNNError", "FRNNShard", "shard_partition", "PATH_AUTO", "PATH_GRID", "PATH_BRUTE", "PATH_BRUTE_TC",
           "library_path", "load_library"]

PATH_AUTO, PATH_GRID, PATH_BRUTE, PATH_BRUTE_TC = 0, 1, 2, 3
PATH_NAMES = {PATH_AUTO: "auto", PATH_GRID: "grid", PATH_BRUTE: "brute", PATH_BRUTE_TC: "brute_tc"}

_OK, _ERR_INVALID, _ERR_OOM, _ERR_CUDA, _ERR_TIMEOUT, _ERR_NODEV, _ERR_STATE, _ERR_COMM = range(8)

_HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None


def library_path() -> str:
    """The engine library: FRNN_B200_LIBRARY if set (an alternate build, e.g.
    with other launch-policy macros), else the in-tree build."""
    return os.environ.get("FRNN_B200_LIBRARY") or os.path.join(_HERE, "libfrnn_b200.so")


class FRNNError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def load_library() -> ctypes.CDLL:
    """Load libfrnn_b200.so (built by pure_cuda-c-_frnn_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing; build it with pure_cuda-c-_frnn_b200/build.py")
    lib = ctypes.CDLL(path)
    P, I, F, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
    sig = {
        "frnn_create": (I, [I, I, ctypes.POINTER(P)]),
        "frnn_destroy": (I, [P]),
        "frnn_search_gpu": (I, [P, P, I, I, I, F, ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_search_gpu_async": (I, [P, P, I, I, I, F, ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_search_gpu_part": (I, [P, P, I, I, I, F, I, I, ctypes.POINTER(I), ctypes.POINTER(P),
                                     ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_search_gpu_queries": (I, [P, P, I, P, I, I, I, F, ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_build_grid": (I, [P, P, I, I, F]),
        "frnn_query_grid": (I, [P, P, I, I, ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_search": (I, [P, P, L, I, F, P, P]),
        "frnn_search_host_soa": (I, [P, P, I, I, I, F, P, P]),
        "frnn_get_results": (I, [P, I, I, P, P]),
        "frnn_status_string": (ctypes.c_char_p, [I]),
        "frnn_last_error": (ctypes.c_char_p, [P]),
        "frnn_set_stream": (I, [P, P]),
        "frnn_set_path": (I, [P, I]),
        "frnn_last_plan": (I, [P, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(L)]),
        "frnn_set_timing": (I, [P, I]),
        "frnn_last_stage_times": (I, [P, ctypes.POINTER(F), I]),
        "frnn_launch_count": (I, [P, ctypes.POINTER(L)]),
        "frnn_set_option": (I, [P, I, L]),
        "frnn_last_grid_axes": (I, [P, ctypes.POINTER(I)]),
        "frnn_last_overflow": (I, [P, ctypes.POINTER(I), P, I]),
        "frnn_shard_unique_id": (I, [P]),
        "frnn_shard_create": (I, [P, I, I, P, ctypes.POINTER(P)]),
        "frnn_shard_destroy": (I, [P]),
        "frnn_shard_set_timeout": (I, [P, ctypes.c_double]),
        "frnn_shard_set_option": (I, [P, I, L]),
        "frnn_search_sharded": (I, [P, I, P, I, I, I, F, ctypes.POINTER(P), ctypes.POINTER(P)]),
        "frnn_shard_last_stats": (I, [P, ctypes.POINTER(F), I, ctypes.POINTER(L), ctypes.POINTER(L),
                                      ctypes.POINTER(I)]),
        "frnn_shard_partition": (I, [P, P, L, I, I, P]),
        "frnn_shard_tc_partition": (I, [I, I, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _raise(lib, eng, st: int, where: str):
    msg = ""
    if eng:
        m = lib.frnn_last_error(eng)
        msg = m.decode() if m else ""
    text = f"{where}: {lib.frnn_status_string(st).decode()}" + (f" ({msg})" if msg else "")
    if st == _ERR_INVALID:
        raise ValueError(text)
    if st == _ERR_OOM:
        raise MemoryError(text)
    raise FRNNError(st, text)


class FRNNEngine:
    """Fixed-radius K-nearest-neighbour engine (self-query).

    Mirrors the reference class FRNNEngine (python_interface/frnn_engine.h:9-55):
    the constructor takes ``max_points``; ``search`` takes a flat row-major host
    array of ``max_points * dim`` floats; ``search_gpu`` takes a raw device
    pointer to SoA data and returns raw device pointers to engine-owned SoA
    results, valid until the next call; ``get_results`` copies them back.

    Result rows are ascending by (squared distance, index); unused slots hold
    index -1 and distance radius**2.
    """

    def __init__(self, max_points: int, device: int = -1):
        self._lib = load_library()
        self._eng = ctypes.c_void_p()
        st = self._lib.frnn_create(int(max_points), int(device), ctypes.byref(self._eng))
        if st != _OK:
            _raise(self._lib, None, st, "FRNNEngine")
        self.max_points = int(max_points)

    # -- lifetime -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_eng", None):
            self._lib.frnn_destroy(self._eng)
            self._eng = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st: int, where: str):
        if st != _OK:
            _raise(self._lib, self._eng, st, where)

    # -- reference surface ------------------------------------------------------
    def search(self, points, K: int, radius: float):
        """Host path (frnn_engine.cu:104-193): ``points`` is a flat row-major
        sequence of max_points*dim floats; returns (idxs, dists) as flat
        row-major lists [q*K + k]."""
        idx, dist = self.search_arrays(points, K, radius)
        return idx.ravel().tolist(), dist.ravel().tolist()

    def search_gpu(self, dev_ptr: int, N: int, dim: int, K: int, radius: float):
        """Device path (frnn_engine.cu:195-250): SoA float32 device pointer in,
        (idx_ptr, dist_ptr) to engine-owned SoA [k*N + q] results out."""
        pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
        st = self._lib.frnn_search_gpu(self._eng, ctypes.c_void_p(int(dev_ptr)), int(N), int(dim),
                                       int(K), float(radius), ctypes.byref(pi), ctypes.byref(pd))
        self._check(st, "search_gpu")
        return int(pi.value), int(pd.value)

    def get_results(self, N: int, K: int):
        """Copy the last results to the host in SoA order [k*N + q]
        (frnn_engine.cu:252-258); returns (idxs, dists) lists."""
        idx, dist = self.get_results_arrays(N, K)
        return idx.ravel().tolist(), dist.ravel().tolist()

    # -- array variants (no reference counterpart) ----------------------------
    def search_arrays(self, points, K: int, radius: float):
        """Like ``search`` but returns numpy arrays of shape (N, K)."""
        pts = np.ascontiguousarray(np.asarray(points, dtype=np.float32).ravel())
        N = self.max_points
        if pts.size == 0 or pts.size % N:
            raise ValueError("points must hold max_points * dim values")
        idx = np.empty((N, int(K)), dtype=np.int32)
        dist = np.empty((N, int(K)), dtype=np.float32)
        st = self._lib.frnn_search(self._eng, pts.ctypes.data, pts.size, int(K), float(radius),
                                   idx.ctypes.data, dist.ctypes.data)
        self._check(st, "search")
        return idx, dist

    def search_soa_host(self, points_soa: np.ndarray, K: int, radius: float,
                        out_idx: np.ndarray | None = None, out_dist: np.ndarray | None = None):
        """Host SoA (D, N) float32 in; SoA (K, N) results out.  Buffers may be
        pinned (e.g. torch pin_memory().numpy()) for full-speed copies."""
        p = np.asarray(points_soa)
        if p.dtype != np.float32 or p.ndim != 2 or not p.flags.c_contiguous:
            raise ValueError("points_soa must be a C-contiguous float32 (D, N) array")
        D, N = p.shape
        if out_idx is None:
            out_idx = np.empty((int(K), N), dtype=np.int32)
        if out_dist is None:
            out_dist = np.empty((int(K), N), dtype=np.float32)
        for a, dt in ((out_idx, np.int32), (out_dist, np.float32)):
            if a.dtype != dt or a.shape != (int(K), N) or not a.flags.c_contiguous:
                raise ValueError("output arrays must be C-contiguous (K, N)")
        st = self._lib.frnn_search_host_soa(self._eng, p.ctypes.data, N, D, int(K), float(radius),
                                            out_idx.ctypes.data, out_dist.ctypes.data)
        self._check(st, "search_soa_host")
        return out_idx, out_dist

    def get_results_arrays(self, N: int, K: int):
        idx = np.empty((int(K), int(N)), dtype=np.int32)
        dist = np.empty((int(K), int(N)), dtype=np.float32)
        st = self._lib.frnn_get_results(self._eng, int(N), int(K), idx.ctypes.data, dist.ctypes.data)
        self._check(st, "get_results")
        return idx, dist

    def search_gpu_async(self, dev_ptr: int, N: int, dim: int, K: int, radius: float):
        pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
        st = self._lib.frnn_search_gpu_async(self._eng, ctypes.c_void_p(int(dev_ptr)), int(N),
                                             int(dim), int(K), float(radius), ctypes.byref(pi),
                                             ctypes.byref(pd))
        self._check(st, "search_gpu_async")
        return int(pi.value), int(pd.value)

    def search_gpu_queries(self, points_ptr: int, N: int, queries_ptr: int, M: int, dim: int, K: int,
                           radius: float):
        """A separate query set (frnn_search_gpu_queries): M SoA queries at
        ``queries_ptr`` against the N SoA points at ``points_ptr``.  Returns
        device pointers to SoA ``[k*M + q]`` results (engine-owned);
        ``get_results(M, K)`` copies them."""
        pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self._lib.frnn_search_gpu_queries(self._eng, ctypes.c_void_p(int(points_ptr)), int(N),
                                                      ctypes.c_void_p(int(queries_ptr)), int(M), int(dim),
                                                      int(K), float(radius), ctypes.byref(pi),
                                                      ctypes.byref(pd)),
                    "search_gpu_queries")
        return pi.value, pd.value

    def build_grid(self, points_ptr: int, N: int, dim: int, radius: float) -> None:
        """Build the search structure for N SoA points once (frnn_build_grid);
        query sets then go through ``query_grid``.  Any other search discards it."""
        self._check(self._lib.frnn_build_grid(self._eng, ctypes.c_void_p(int(points_ptr)), int(N), int(dim),
                                              float(radius)),
                    "build_grid")

    def query_grid(self, queries_ptr: int, M: int, K: int):
        """Search M SoA queries against the built grid (frnn_query_grid);
        returns device pointers to SoA ``[k*M + q]`` results."""
        pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self._lib.frnn_query_grid(self._eng, ctypes.c_void_p(int(queries_ptr)), int(M), int(K),
                                              ctypes.byref(pi), ctypes.byref(pd)),
                    "query_grid")
        return pi.value, pd.value

    def search_gpu_part(self, dev_ptr: int, N: int, dim: int, K: int, radius: float, part: int,
                        nparts: int):
        """One of ``nparts`` slices of the search (frnn_search_gpu_part): returns
        ``(n_rows, row_ids_ptr, idx_ptr, dist_ptr)``; row j of the SoA results
        (``[k*n_rows + j]``) is query ``row_ids[j]``.  Device pointers are
        engine-owned and valid until the next call."""
        n = ctypes.c_int()
        pr, pi, pd = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self._lib.frnn_search_gpu_part(self._eng, ctypes.c_void_p(int(dev_ptr)), int(N),
                                                   int(dim), int(K), float(radius), int(part),
                                                   int(nparts), ctypes.byref(n), ctypes.byref(pr),
                                                   ctypes.byref(pi), ctypes.byref(pd)),
                    "search_gpu_part")
        return n.value, pr.value or 0, pi.value or 0, pd.value or 0

    def set_stream(self, stream: int) -> None:
        self._check(self._lib.frnn_set_stream(self._eng, ctypes.c_void_p(int(stream))), "set_stream")

    def set_path(self, path: int | str) -> None:
        if isinstance(path, str):
            path = {v: k for k, v in PATH_NAMES.items()}[path]
        self._check(self._lib.frnn_set_path(self._eng, int(path)), "set_path")

    OPT_DIRECT_OUTPUT_MAX_BYTES = 1
    OPT_GRID_AXES = 2
    OPT_LIST_SEARCH = 3
    OPT_TEST_STALL = 4
    OPT_DEVICE_PLAN = 5
    OPT_TC_SYMMETRIC = 6
    TEST_STALL_OFF, TEST_STALL_SCAN, TEST_STALL_TC_FILTER = 0, 1, 2
    GRID_AXES_AUTO, GRID_AXES_LEADING, GRID_AXES_PRINCIPAL = 0, 1, 2
    LIST_SEARCH_AUTO, LIST_SEARCH_ALWAYS, LIST_SEARCH_NEVER = 0, 1, 2

    def set_option(self, option: int, value: int) -> None:
        self._check(self._lib.frnn_set_option(self._eng, int(option), int(value)), "set_option")

    STAGES = ("bbox", "hash", "scan", "scatter", "search", "unpermute", "brute", "collect", "emit",
              "tc_prep", "tc_filter", "tc_rerank")

    def set_timing(self, enable: bool) -> None:
        self._check(self._lib.frnn_set_timing(self._eng, int(bool(enable))), "set_timing")

    def stage_times(self) -> dict:
        """Milliseconds per stage of the last search (timing must be on)."""
        n = len(self.STAGES)
        buf = (ctypes.c_float * n)()
        self._check(self._lib.frnn_last_stage_times(self._eng, buf, n), "stage_times")
        return {k: float(v) for k, v in zip(self.STAGES, buf) if v >= 0}

    def last_overflow(self, max_ids: int = 1 << 24) -> np.ndarray:
        """Original indices of the queries of the last whole search whose
        candidate list overflowed and were searched again by the fallback
        pass (sorted ascending)."""
        n = ctypes.c_int()
        self._check(self._lib.frnn_last_overflow(self._eng, ctypes.byref(n), None, 0), "last_overflow")
        m = min(int(n.value), int(max_ids))
        out = np.empty(m, dtype=np.int32)
        if m:
            self._check(self._lib.frnn_last_overflow(self._eng, ctypes.byref(n), out.ctypes.data, m),
                        "last_overflow")
        return np.sort(out)

    def launch_count(self) -> int:
        n = ctypes.c_int64()
        self._check(self._lib.frnn_launch_count(self._eng, ctypes.byref(n)), "launch_count")
        return int(n.value)

    def last_plan(self) -> dict:
        p, g, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        self._check(self._lib.frnn_last_plan(self._eng, ctypes.byref(p), ctypes.byref(g),
                                             ctypes.byref(c)), "last_plan")
        ax = ctypes.c_int()
        self._check(self._lib.frnn_last_grid_axes(self._eng, ctypes.byref(ax)), "last_plan")
        return {"path": PATH_NAMES.get(p.value, str(p.value)), "grid_dims": g.value, "cells": c.value,
                "axes": "principal" if ax.value == self.GRID_AXES_PRINCIPAL else "leading"}


def shard_partition(tile_work, tile_start, N: int, nparts: int) -> np.ndarray:
    """The cut points a sharded search applies (frnn_shard_partition, host
    code): query-order tiles starting at ``tile_start`` with estimated work
    ``tile_work``; returns ``bounds[0..nparts]``, slice r = [bounds[r], bounds[r+1])."""
    lib = load_library()
    w = np.ascontiguousarray(tile_work, dtype=np.uint64)
    t = np.ascontiguousarray(tile_start, dtype=np.int32)
    if w.shape != t.shape or w.ndim != 1:
        raise ValueError("tile_work and tile_start must be 1-D of the same length")
    out = np.empty(int(nparts) + 1, dtype=np.int32)
    st = lib.frnn_shard_partition(w.ctypes.data, t.ctypes.data, len(w), int(N), int(nparts), out.ctypes.data)
    if st != _OK:
        _raise(lib, None, st, "shard_partition")
    return out


def shard_tc_partition(N: int, nparts: int) -> np.ndarray:
    """The cut points of a sharded tensor-core search that shares the
    symmetric filter (frnn_shard_tc_partition, host code): bounds[0..nparts],
    rank r owns queries [bounds[r], bounds[r+1])."""
    lib = load_library()
    out = np.empty(int(nparts) + 1, dtype=np.int32)
    st = lib.frnn_shard_tc_partition(int(N), int(nparts), out.ctypes.data)
    if st != _OK:
        _raise(lib, None, st, "shard_tc_partition")
    return out


class FRNNShard:
    """One rank of a query-sharded search (frnn_shard_*): ``engine`` (on this
    process's GPU) joined to the other ranks' engines by an NCCL communicator.

    Every rank constructs it with the same ``uid`` (``FRNNShard.unique_id()``
    on one rank, shared over any host channel) and then calls ``search`` with
    the same arguments; the root passes its cloud and receives device pointers
    to the [K, N] results, valid until the next call."""

    ID_BYTES = 128
    STAGES = ("build", "header", "broadcast", "search", "gather")

    @staticmethod
    def unique_id() -> bytes:
        lib = load_library()
        buf = (ctypes.c_ubyte * FRNNShard.ID_BYTES)()
        st = lib.frnn_shard_unique_id(buf)
        if st != _OK:
            _raise(lib, None, st, "shard unique_id")
        return bytes(buf)

    def __init__(self, engine: "FRNNEngine", nranks: int, rank: int, uid: bytes):
        if len(uid) != self.ID_BYTES:
            raise ValueError(f"uid must be {self.ID_BYTES} bytes")
        self._engine = engine
        self._lib = engine._lib
        self._sh = ctypes.c_void_p()
        buf = (ctypes.c_ubyte * self.ID_BYTES).from_buffer_copy(uid)
        st = self._lib.frnn_shard_create(engine._eng, int(nranks), int(rank), buf, ctypes.byref(self._sh))
        if st != _OK:
            _raise(self._lib, engine._eng, st, "shard create")
        self.nranks, self.rank = int(nranks), int(rank)

    def close(self) -> None:
        if getattr(self, "_sh", None):
            self._lib.frnn_shard_destroy(self._sh)
            self._sh = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_timeout(self, seconds: float) -> None:
        st = self._lib.frnn_shard_set_timeout(self._sh, float(seconds))
        if st != _OK:
            _raise(self._lib, self._engine._eng, st, "shard set_timeout")

    OPT_CHUNKS, OPT_COMM_PRIORITY, OPT_TC_SYMMETRIC = 1, 2, 3

    def set_option(self, option: int, value: int) -> None:
        st = self._lib.frnn_shard_set_option(self._sh, int(option), int(value))
        if st != _OK:
            _raise(self._lib, self._engine._eng, st, "shard set_option")

    def search(self, root: int, dev_ptr: int, N: int, dim: int, K: int, radius: float):
        """frnn_search_sharded: (idx_ptr, dist_ptr) of the [K, N] results on
        the root, (0, 0) on the other ranks."""
        pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
        st = self._lib.frnn_search_sharded(self._sh, int(root), ctypes.c_void_p(int(dev_ptr or 0)), int(N),
                                           int(dim), int(K), float(radius), ctypes.byref(pi), ctypes.byref(pd))
        if st != _OK:
            _raise(self._lib, self._engine._eng, st, "search_sharded")
        return pi.value or 0, pd.value or 0

    def last_stats(self) -> dict:
        n = len(self.STAGES)
        ms = (ctypes.c_float * n)()
        bb, gb, rows = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        st = self._lib.frnn_shard_last_stats(self._sh, ms, n, ctypes.byref(bb), ctypes.byref(gb),
                                             ctypes.byref(rows))
        if st != _OK:
            _raise(self._lib, self._engine._eng, st, "shard last_stats")
        return {"stage_ms": {k: float(v) for k, v in zip(self.STAGES, ms) if v >= 0},
                "broadcast_bytes": int(bb.value), "gather_bytes": int(gb.value), "rows": int(rows.value)}
