"""The allocation-free search entry point (cvs_fused_topk_noalloc).

It exists for callers that cannot allocate device memory themselves -- a host
application that owns the device-memory budget and does not let plugins call
cudaMalloc, a serving loop that cannot take cudaMalloc's synchronisation, a
language binding without a device allocator. It runs the same kernels as
cvs_fused_topk with the candidate lists in a fixed array inside the library.

This test calls both entry points through the C ABI (ctypes) on the same inputs
and checks that the allocation-free one returns the same ids and scores as the
other and as the CPU oracle, twice in a row (the second call reuses the array
the first call left behind). It is
named so pytest collects it after every other test file.
"""

import ctypes
from pathlib import Path

import pytest
import torch

from cases import make
from helpers import assert_topk_exact
from oracle import exact_topk

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "cuda-vector-search_b200" / "cuda_vector_search" / "libcvs_b200.so"


def _lib():
    lib = ctypes.CDLL(str(LIB))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.cvs_fused_topk.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, vp, ctypes.c_size_t, i32, i32, vp, vp]
    lib.cvs_fused_topk.restype = i32
    lib.cvs_fused_topk_noalloc.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, i32, vp]
    lib.cvs_fused_topk_noalloc.restype = i32
    lib.cvs_fused_topk_workspace_size.argtypes = [i64, i64, i32, i32, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
    lib.cvs_fused_topk_workspace_size.restype = i32
    lib.cvs_last_error.restype = ctypes.c_char_p
    return lib


def _with_workspace(lib, q, x, k, stream):
    b, n, d_pad = q.shape[0], x.shape[0], x.shape[1]
    nbytes = ctypes.c_size_t(0)
    assert lib.cvs_fused_topk_workspace_size(b, n, d_pad, k, 0, 0, ctypes.byref(nbytes)) == 0
    ws = torch.empty(max(256, nbytes.value), dtype=torch.uint8, device=q.device)
    v = torch.empty((b, k), dtype=torch.float32, device=q.device)
    i = torch.empty((b, k), dtype=torch.int64, device=q.device)
    st = lib.cvs_fused_topk(q.data_ptr(), b, x.data_ptr(), n, d_pad, k, 0, v.data_ptr(), i.data_ptr(),
                            ws.data_ptr(), ws.numel(), 0, 0, None, stream)
    assert st == 0, lib.cvs_last_error()
    torch.cuda.synchronize()
    return v.cpu(), i.cpu()


def _no_alloc(lib, q, x, k, stream, plan_chunks=0, expect=0):
    b, n, d_pad = q.shape[0], x.shape[0], x.shape[1]
    # Outputs come from the caller; the entry point itself allocates nothing.
    v = torch.full((b, k), float("nan"), dtype=torch.float32, device=q.device)
    i = torch.full((b, k), -7, dtype=torch.int64, device=q.device)
    st = lib.cvs_fused_topk_noalloc(q.data_ptr(), b, x.data_ptr(), n, d_pad, k, 0, v.data_ptr(), i.data_ptr(),
                                    plan_chunks, stream)
    assert st == expect, lib.cvs_last_error()
    torch.cuda.synchronize()
    return v.cpu(), i.cpu()


# (300000, 64, 256, 256): the automatic plan needs more than the built-in
# scratch, so the entry point plans fewer corpus segments. (20000, 128, 1, 1024):
# a single query with the largest k (tcgen05 path, many long buffer lists).
@pytest.mark.parametrize("n,d,b,k", [(20000, 768, 256, 10), (30000, 384, 40, 100), (20000, 768, 1, 10),
                                     (300000, 64, 256, 256), (20000, 128, 1, 1024)])
def test_no_alloc_matches_workspace_entry_point(n, d, b, k):
    assert torch.cuda.is_available()
    lib = _lib()
    x, q = make(n, d, b, seed=n + b + k)
    x, q = x.cuda(), q.cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref_v, ref_i = _with_workspace(lib, q, x, k, stream)
    x32, q32 = x.float().cpu().numpy(), q.float().cpu().numpy()
    ov, oi = exact_topk(q32, x32, min(k + 1, n))
    for _ in range(2):  # the second call starts from the first call's leftovers
        v, i = _no_alloc(lib, q, x, k, stream)
        assert_topk_exact(v.numpy(), i.numpy(), q32, x32, ov, oi, k)
        assert torch.equal(i, ref_i)
        assert torch.allclose(v, ref_v, atol=1e-3, rtol=0)


def test_no_alloc_rejects_an_explicit_plan_that_does_not_fit():
    """An explicit segment count is taken as given: if its lists exceed the
    built-in scratch the call fails (no re-planning); automatic planning of the
    same problem fits and matches the oracle."""
    lib = _lib()
    x, q = make(300000, 64, 256, seed=5)
    x, q = x.cuda(), q.cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _no_alloc(lib, q, x, 256, stream, plan_chunks=200, expect=3)
    assert b"built-in scratch" in lib.cvs_last_error()
    v, i = _no_alloc(lib, q, x, 256, stream)
    x32, q32 = x.float().cpu().numpy(), q.float().cpu().numpy()
    ov, oi = exact_topk(q32, x32, 257)
    assert_topk_exact(v.numpy(), i.numpy(), q32, x32, ov, oi, 256)


def test_no_alloc_rejects_oversize_problem():
    lib = _lib()
    # Even one corpus segment needs b * 2 lists * 2048 slots * 8 bytes = 32 MiB.
    x, q = make(20000, 64, 1024, seed=1)
    x, q = x.cuda(), q.cuda()
    b, n = q.shape[0], x.shape[0]
    v = torch.empty((b, 1024), dtype=torch.float32, device="cuda")
    i = torch.empty((b, 1024), dtype=torch.int64, device="cuda")
    st = lib.cvs_fused_topk_noalloc(q.data_ptr(), b, x.data_ptr(), n, 64, 1024, 0, v.data_ptr(), i.data_ptr(), 0,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 3  # CVS_ERR_WORKSPACE
    assert b"built-in scratch" in lib.cvs_last_error()
