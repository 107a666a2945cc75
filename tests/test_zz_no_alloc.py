"""The allocation-free entry point frnn_search_gpu_noalloc, through the C ABI.

It exists for callers that cannot allocate device memory while they search
(their framework's pool owns the device memory, or allocation stalls are not
allowed in their loop).  It must return exactly what frnn_search_gpu returns
for the same input; two calls in a row check that the fixed scratch it shares
between calls does not carry state from one call into the next.  This file
sorts last so a failure here never hides the rest of the suite.
"""

import ctypes

import numpy as np
import pytest

from frnn_cuda import datagen
from parity import assert_bit_exact

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def noalloc():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frnn_cuda
    lib = frnn_cuda.load_library()
    fn = lib.frnn_search_gpu_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return frnn_cuda, fn


def reference_results(frnn_cuda, soa, K, r):
    D, N = soa.shape
    eng = frnn_cuda.FRNNEngine(max_points=N)
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    eng.search_gpu(t.data_ptr(), N, D, K, r)
    return eng.get_results_arrays(N, K)


def noalloc_results(fn, soa, K, r):
    D, N = soa.shape
    t = torch.from_numpy(np.ascontiguousarray(soa)).cuda()
    oi = torch.empty((K, N), dtype=torch.int32, device="cuda")
    od = torch.empty((K, N), dtype=torch.float32, device="cuda")
    st = fn(t.data_ptr(), N, D, K, r, oi.data_ptr(), od.data_ptr(), None)
    assert st == 0, st
    return oi.cpu().numpy(), od.cpu().numpy()


def test_noalloc_matches_search_gpu_two_calls(noalloc, oracle_mod):
    frnn_cuda, fn = noalloc
    # call 1: D=3 mixture, grid path; call 2: D=12 low-rank, first-coordinate grid
    cases = [("mixture", 60000, 3, 32), ("lowrank4", 50000, 12, 16)]
    for kind, N, D, K in cases:
        pts = datagen.generate(kind, N, D, seed=N + D)
        soa = datagen.soa(pts)
        r = datagen.calibrate_radius(pts, 0.75 * K, sample=256)
        ri, rd = reference_results(frnn_cuda, soa, K, r)
        ni, nd = noalloc_results(fn, soa, K, r)
        assert_bit_exact(ni, nd, ri, rd, f"noalloc {kind} D={D}")
        oi, od, _ = oracle_mod.search(soa, K, r)
        assert_bit_exact(ni, nd, oi, od, f"noalloc vs oracle {kind} D={D}")


# Every branch of the entry point, in an order that runs a grid with many
# cells before grids with few, so stale scratch from an earlier call would
# show: (kind, N, D, K, radius scale relative to the calibrated one).
BRANCHES = [
    ("uniform", 65536, 2, 8, 0.3),     # fine 2-D grid near the 2^19-cell cap
    ("uniform", 5000, 3, 16, 1.0),     # N*N*D <= 4e8: brute force
    ("lowrank6", 40000, 16, 128, 1.0),  # D = 16 (four float4 per row), K = 128
    ("uniform", 30000, 1, 4, 1.0),     # D = 1
    ("uniform", 30000, 3, 8, 40.0),    # radius so large that no grid helps: brute force
    ("mixture", 65536, 14, 33, 1.0),   # D in 13..16, K > 32
    ("uniform", 20000, 2, 5, 1.0),     # a small grid after the large ones
]


def test_noalloc_every_branch_vs_oracle(noalloc, oracle_mod):
    frnn_cuda, fn = noalloc
    for kind, N, D, K, scale in BRANCHES:
        pts = datagen.generate(kind, N, D, seed=7 * N + D)
        soa = datagen.soa(pts)
        r = scale * datagen.calibrate_radius(pts, max(1.0, 0.75 * K), sample=128)
        ni, nd = noalloc_results(fn, soa, K, r)
        oi, od, _ = oracle_mod.search(soa, K, r)
        assert_bit_exact(ni, nd, oi, od, f"noalloc {kind} N={N} D={D} K={K} x{scale}")
        ri, rd = reference_results(frnn_cuda, soa, K, r)
        assert_bit_exact(ni, nd, ri, rd, f"noalloc vs search_gpu {kind} N={N} D={D}")


def test_noalloc_rejects_nonfinite_points(noalloc):
    frnn_cuda, fn = noalloc
    pts = datagen.generate("uniform", 40000, 3, seed=5)
    pts[1234, 1] = np.nan
    t = torch.from_numpy(datagen.soa(pts)).cuda()
    o = torch.empty(8 * 40000, device="cuda")
    assert fn(t.data_ptr(), 40000, 3, 8, 0.01, o.data_ptr(), o.data_ptr(), None) == 1


def test_noalloc_rejects_sizes_beyond_its_limits(noalloc):
    frnn_cuda, fn = noalloc
    t = torch.zeros(17 * 70000, device="cuda")
    o = torch.empty(4 * 70000, device="cuda")
    assert fn(t.data_ptr(), 70000, 3, 4, 0.1, o.data_ptr(), o.data_ptr(), None) == 1  # N
    assert fn(t.data_ptr(), 1000, 17, 4, 0.1, o.data_ptr(), o.data_ptr(), None) == 1   # dim
    assert fn(t.data_ptr(), 1000, 3, 129, 0.1, o.data_ptr(), o.data_ptr(), None) == 1  # K
