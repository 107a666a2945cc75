"""The C-ABI library loads and exports every entry point that
include/frnn_b200.h declares; argument checking that needs no GPU."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "frnn_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(frnn_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    fns = declared_functions()
    for name in ("frnn_create", "frnn_destroy", "frnn_search_gpu", "frnn_search", "frnn_get_results"):
        assert name in fns


def test_library_exports_every_declared_symbol():
    import frnn_cuda
    lib = frnn_cuda.load_library()
    missing = [f for f in declared_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_status_strings():
    import frnn_cuda
    lib = frnn_cuda.load_library()
    assert lib.frnn_status_string(0) == b"ok"
    assert lib.frnn_status_string(1) == b"invalid argument"
    assert lib.frnn_status_string(99) == b"unknown status"


def test_create_argument_checks_without_device():
    import frnn_cuda
    lib = frnn_cuda.load_library()
    h = ctypes.c_void_p()
    assert lib.frnn_create(0, -1, ctypes.byref(h)) == 1  # bad max_points
    assert lib.frnn_create(10, -1, None) == 1             # null out pointer
    assert lib.frnn_destroy(None) == 0


def test_null_engine_is_rejected():
    import frnn_cuda
    lib = frnn_cuda.load_library()
    pi, pd = ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.frnn_search_gpu(None, None, 1, 3, 1, 1.0, ctypes.byref(pi), ctypes.byref(pd)) == 1
    assert lib.frnn_get_results(None, 1, 1, None, None) == 1
    assert lib.frnn_set_path(None, 0) == 1


def test_no_device_reported_on_cpu_host():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import frnn_cuda
    with pytest.raises(frnn_cuda.FRNNError) as ei:
        frnn_cuda.FRNNEngine(100)
    assert ei.value.status == 5
