"""The C ABI library loads without a GPU, exports every function include/cvs.h
declares, and enforces its argument contracts before touching a device."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "cuda-vector-search_b200" / "cuda_vector_search" / "libcvs_b200.so"
HEADER = ROOT / "include" / "cvs.h"


@pytest.fixture(scope="module")
def lib():
    assert LIB.exists(), "build first: python cuda-vector-search_b200/build.py"
    lib = ctypes.CDLL(str(LIB))
    lib.cvs_last_error.restype = ctypes.c_char_p
    return lib


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:cvs_status|int|const char\*)\s+(cvs_\w+)\s*\(", text, re.M)))


def test_header_declares_the_search_surface():
    names = declared_functions()
    for must in ("cvs_fused_topk", "cvs_fused_topk_workspace_size", "cvs_scores", "cvs_ingest",
                 "cvs_merge_lists", "cvs_last_error", "cvs_poll_device_error"):
        assert must in names


def test_every_declared_function_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/cvs.h but not exported"


def test_version_and_padding(lib):
    assert lib.cvs_abi_version() == 1
    for d, want in [(1, 64), (64, 64), (65, 128), (96, 128), (768, 768), (1000, 1024)]:
        assert lib.cvs_pad_width(d) == want


def test_workspace_size_rejects_bad_shapes(lib):
    n = ctypes.c_size_t(0)
    i64, i32 = ctypes.c_int64, ctypes.c_int
    f = lib.cvs_fused_topk_workspace_size
    f.argtypes = [i64, i64, i32, i32, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
    assert f(4, 1000, 100, 10, 0, 0, ctypes.byref(n)) == 1  # width not a multiple of 64
    assert b"multiple of 64" in lib.cvs_last_error()
    assert f(4, 0, 128, 10, 0, 0, ctypes.byref(n)) == 1  # empty corpus
    assert f(-1, 10, 128, 10, 0, 0, ctypes.byref(n)) == 1
    assert f(0, 10, 128, 10, 0, 0, ctypes.byref(n)) == 0 and n.value == 0  # no queries: nothing to do


def test_fused_topk_contract_errors_before_any_device_use(lib):
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f = lib.cvs_fused_topk
    f.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, vp, ctypes.c_size_t, i32, i32, vp, vp]
    assert f(None, 4, None, 100, 64, 10, 0, None, None, None, 0, 0, 0, None, None) == 1
    assert b"corpus" in lib.cvs_last_error()
    assert f(16, 4, 3, 100, 64, 10, 0, None, None, None, 0, 0, 0, None, None) == 1
    assert b"aligned" in lib.cvs_last_error()


def test_merge_and_ingest_contracts(lib):
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.cvs_merge_lists.argtypes = [vp, vp, i64, i64, i64, i32, vp, vp, vp]
    assert lib.cvs_merge_lists(None, None, 0, 4, 10, 5, None, None, None) == 1
    assert lib.cvs_merge_lists(None, None, 2, 4, 10, 0, None, None, None) == 1
    lib.cvs_merge_lists_strided.argtypes = [vp, i64, vp, i64, i64, i64, i64, i32, vp, vp, vp]
    # strides below b * len would overlap lists
    assert lib.cvs_merge_lists_strided(16, 39, 16, 40, 2, 4, 10, 5, 16, 16, None) == 1
    assert b"stride" in lib.cvs_last_error()
    assert lib.cvs_merge_lists_strided(16, 40, 16, 40, 2, 4, 10, 2000, 16, 16, None) == 1  # k too large
    lib.cvs_ingest.argtypes = [vp, i32, i64, i32, i64, i32, i32, vp, vp]
    assert lib.cvs_ingest(None, 0, 0, 8, 8, 64, 1, None, None) == 0  # zero rows: nothing to do
    assert lib.cvs_ingest(None, 0, 5, 8, 8, 64, 1, None, None) == 1
    assert lib.cvs_ingest(16, 0, 5, 100, 100, 96, 1, 16, None) == 1  # d_pad not a multiple of 64
    assert lib.cvs_ingest(16, 9, 5, 64, 64, 64, 1, 32, None) == 1  # unknown dtype
    assert b"dtype" in lib.cvs_last_error()


def test_search_contract_errors_before_any_device_use(lib):
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f = lib.cvs_search
    f.argtypes = [vp, i32, i64, i32, i64, i32, vp, i64, i32, i32, i64, vp, vp, vp, ctypes.c_size_t, vp]
    assert f(None, 0, 4, 64, 64, 1, 16, 100, 64, 10, 0, 16, 16, 256, 1 << 20, None) == 1
    assert b"queries" in lib.cvs_last_error()
    assert f(16, 0, 4, 100, 100, 1, 16, 100, 64, 10, 0, 16, 16, 256, 1 << 20, None) == 1  # wider than the corpus
    assert b"exceeds" in lib.cvs_last_error()
    assert f(16, 7, 4, 64, 64, 1, 16, 100, 64, 10, 0, 16, 16, 256, 1 << 20, None) == 1  # unknown dtype
    assert f(16, 0, 4, 64, 32, 1, 16, 100, 64, 10, 0, 16, 16, 256, 1 << 20, None) == 1  # stride < width
    assert f(16, 0, 0, 64, 64, 1, 16, 100, 64, 10, 0, 16, 16, 256, 1 << 20, None) == 0  # no queries: nothing to do
    n = ctypes.c_size_t(0)
    g = lib.cvs_search_workspace_size
    g.argtypes = [i64, i64, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
    assert g(4, 1000, 100, 10, ctypes.byref(n)) == 1
    assert g(0, 10, 128, 10, ctypes.byref(n)) == 0 and n.value == 0


def test_stall_hook_rejects_out_of_range_limits(lib):
    lib.cvs_debug_stall_next_search.argtypes = [ctypes.c_int64]
    assert lib.cvs_debug_stall_next_search(10) == 1
    assert lib.cvs_debug_stall_next_search(1 << 50) == 1
