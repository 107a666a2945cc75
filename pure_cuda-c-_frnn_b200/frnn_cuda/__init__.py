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

__all__ = ["FRNNEngine", "FRNNError", "PATH_AUTO", "PATH_GRID", "PATH_BRUTE", "PATH_BRUTE_TC",
           "library_path", "load_library"]

PATH_AUTO, PATH_GRID, PATH_BRUTE, PATH_BRUTE_TC = 0, 1, 2, 3
PATH_NAMES = {PATH_AUTO: "auto", PATH_GRID: "grid", PATH_BRUTE: "brute", PATH_BRUTE_TC: "brute_tc"}

_OK, _ERR_INVALID, _ERR_OOM, _ERR_CUDA, _ERR_TIMEOUT, _ERR_NODEV, _ERR_STATE = range(7)

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
