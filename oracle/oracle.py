"""ctypes bindings of the parity checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
its reference arm) use this module; the engine never imports it.

  * liboracle.so            -- CPU restatement of the reference (frnn_oracle.cpp)
  * _ref/libfrnn_ref.so     -- the reference engine compiled from its own sources
                               (Makefile target ``ref``); needs a GPU to run.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfrnn_ref.so")

ORDER_ENGINE, ORDER_CHAIN, ORDER_AOS3, ORDER_BF4 = 0, 1, 2, 3
PATH_NAMES = {0: "bf_small", 1: "grid_aos3", 2: "grid_nd", 3: "firstd", 4: "bf_fallback"}

_oracle = None
_ref = None


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and the reference library when ``ref``)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        P, I, F, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong
        L.oracle_ref_plan.argtypes = [I, I, I, F, ctypes.POINTER(I), ctypes.POINTER(I),
                                      ctypes.POINTER(I), ctypes.POINTER(LL)]
        L.oracle_search.argtypes = [P, I, I, I, F, I, I, P, P, ctypes.POINTER(LL)]
        L.oracle_search_subset.argtypes = [P, I, I, I, F, I, P, I, I, P, P, ctypes.POINTER(LL)]
        L.oracle_search_queries.argtypes = [P, I, P, I, I, I, F, I, I, P, P, ctypes.POINTER(LL)]
        L.oracle_ref_search.argtypes = [P, I, I, I, F, I, P, P, P, ctypes.POINTER(I)]
        L.oracle_pair_d2_f64.argtypes = [P, I, I, P, P, LL, P]
        L.oracle_pair_d2_f32.argtypes = [P, I, I, I, P, P, LL, P]
        for f in ("oracle_ref_plan", "oracle_search", "oracle_search_subset", "oracle_search_queries",
                  "oracle_ref_search", "oracle_pair_d2_f64", "oracle_pair_d2_f32", "oracle_max_threads"):
            getattr(L, f).restype = I
        _oracle = L
    return _oracle


def _soa(pts_soa: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(pts_soa, dtype=np.float32)
    assert a.ndim == 2
    return a


def ref_plan(N: int, D: int, K: int, r: float) -> dict:
    p, g, res, cells = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_longlong()
    st = lib().oracle_ref_plan(N, D, K, r, ctypes.byref(p), ctypes.byref(g), ctypes.byref(res),
                               ctypes.byref(cells))
    assert st == 0
    return {"path": PATH_NAMES[p.value], "grid_dim": g.value, "res": res.value, "cells": cells.value}


def search(pts_soa: np.ndarray, K: int, r: float, order: int = ORDER_ENGINE, threads: int = 0):
    """Exact search, every point a query.  Returns SoA (K, N) idx, dist and the
    number of candidate distances evaluated."""
    p = _soa(pts_soa)
    D, N = p.shape
    idx = np.empty((K, N), np.int32)
    dist = np.empty((K, N), np.float32)
    nc = ctypes.c_longlong()
    st = lib().oracle_search(p.ctypes.data, N, D, K, float(r), order, threads, idx.ctypes.data,
                             dist.ctypes.data, ctypes.byref(nc))
    assert st == 0, st
    return idx, dist, nc.value


def search_subset(pts_soa: np.ndarray, qids: np.ndarray, K: int, r: float,
                  order: int = ORDER_ENGINE, threads: int = 0):
    """Exact search for queries qids against all points; SoA (K, nq) out."""
    p = _soa(pts_soa)
    D, N = p.shape
    q = np.ascontiguousarray(qids, dtype=np.int32)
    idx = np.empty((K, len(q)), np.int32)
    dist = np.empty((K, len(q)), np.float32)
    nc = ctypes.c_longlong()
    st = lib().oracle_search_subset(p.ctypes.data, N, D, K, float(r), order, q.ctypes.data, len(q),
                                    threads, idx.ctypes.data, dist.ctypes.data, ctypes.byref(nc))
    assert st == 0, st
    return idx, dist, nc.value


def search_queries(pts_soa: np.ndarray, q_soa: np.ndarray, K: int, r: float,
                   order: int = ORDER_ENGINE, threads: int = 0):
    """Exact search of a separate query set (SoA (D, M)) against the points
    (SoA (D, N)); SoA (K, M) out."""
    p = _soa(pts_soa)
    q = _soa(q_soa)
    D, N = p.shape
    assert q.shape[0] == D
    M = q.shape[1]
    idx = np.empty((K, M), np.int32)
    dist = np.empty((K, M), np.float32)
    nc = ctypes.c_longlong()
    st = lib().oracle_search_queries(p.ctypes.data, N, q.ctypes.data, M, D, K, float(r), order, threads,
                                     idx.ctypes.data, dist.ctypes.data, ctypes.byref(nc))
    assert st == 0, st
    return idx, dist, nc.value


def ref_search(pts_soa: np.ndarray, K: int, r: float, threads: int = 0):
    """Reference-mode search (reference dispatch, per-path arithmetic and
    domain rule).  Returns idx, dist (K, N), valid mask (N,), path name."""
    p = _soa(pts_soa)
    D, N = p.shape
    idx = np.empty((K, N), np.int32)
    dist = np.empty((K, N), np.float32)
    valid = np.empty(N, np.uint8)
    path = ctypes.c_int()
    st = lib().oracle_ref_search(p.ctypes.data, N, D, K, float(r), threads, idx.ctypes.data,
                                 dist.ctypes.data, valid.ctypes.data, ctypes.byref(path))
    assert st == 0, st
    return idx, dist, valid.astype(bool), PATH_NAMES[path.value]


def pair_d2_f64(pts_soa: np.ndarray, qi: np.ndarray, pj: np.ndarray) -> np.ndarray:
    p = _soa(pts_soa)
    D, N = p.shape
    qi = np.ascontiguousarray(qi, np.int32)
    pj = np.ascontiguousarray(pj, np.int32)
    out = np.empty(len(qi), np.float64)
    assert lib().oracle_pair_d2_f64(p.ctypes.data, N, D, qi.ctypes.data, pj.ctypes.data, len(qi),
                                    out.ctypes.data) == 0
    return out


def pair_d2_f32(pts_soa: np.ndarray, qi: np.ndarray, pj: np.ndarray, order: int = ORDER_ENGINE):
    p = _soa(pts_soa)
    D, N = p.shape
    qi = np.ascontiguousarray(qi, np.int32)
    pj = np.ascontiguousarray(pj, np.int32)
    out = np.empty(len(qi), np.float32)
    assert lib().oracle_pair_d2_f32(p.ctypes.data, N, D, order, qi.ctypes.data, pj.ctypes.data,
                                    len(qi), out.ctypes.data) == 0
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ---- the reference engine, compiled from its sources (needs a GPU) --------------


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} is missing (make -C oracle ref)")
        L = ctypes.CDLL(REF_SO)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.ref_create.argtypes = [I]
        L.ref_create.restype = P
        L.ref_destroy.argtypes = [P]
        L.ref_destroy.restype = None
        L.ref_search_gpu.argtypes = [P, P, I, I, I, F, ctypes.POINTER(ctypes.c_uint64),
                                     ctypes.POINTER(ctypes.c_uint64)]
        L.ref_search_gpu.restype = I
        L.ref_get_results.argtypes = [P, I, I, P, P]
        L.ref_get_results.restype = I
        L.ref_search_host.argtypes = [P, P, I, I, I, F, P, P]
        L.ref_search_host.restype = I
        _ref = L
    return _ref


class RefEngine:
    """The reference FRNNEngine (built from its sources) behind ctypes."""

    def __init__(self, max_points: int):
        self.L = ref_lib()
        self.h = self.L.ref_create(int(max_points))
        if not self.h:
            raise RuntimeError("ref_create failed")
        self.max_points = int(max_points)

    def close(self):
        if self.h:
            self.L.ref_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search_gpu(self, dev_ptr: int, N: int, dim: int, K: int, r: float):
        a, b = ctypes.c_uint64(), ctypes.c_uint64()
        st = self.L.ref_search_gpu(self.h, ctypes.c_void_p(int(dev_ptr)), N, dim, K, float(r),
                                   ctypes.byref(a), ctypes.byref(b))
        if st != 0:
            raise RuntimeError(f"reference search_gpu failed ({st})")
        return a.value, b.value

    def get_results(self, N: int, K: int):
        idx = np.empty((K, N), np.int32)
        dist = np.empty((K, N), np.float32)
        assert self.L.ref_get_results(self.h, N, K, idx.ctypes.data, dist.ctypes.data) == 0
        return idx, dist
