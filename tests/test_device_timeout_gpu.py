"""The device-side failure path, exercised without faulting or hanging the GPU.

Every pipeline wait in the search kernels is bounded; when one runs out the
kernel records a code in the per-device error word, drains what it issued,
frees its tensor memory and returns, and the host reads the code with
cvs_poll_device_error. Here the C ABI's test hook (cvs_debug_stall_next_search)
makes one search's producer claim nothing and shortens its waits to 10^6 SM
clocks (about half a millisecond), so its MMA issuer and drain warps wait on an
iteration log that nothing writes. The test checks that the call returns, that
the poll reports CVS_ERR_DEVICE_TIMEOUT with an iteration-log wait site, and
that the next ordinary search on the same GPU is exact.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import make
from helpers import assert_topk_exact
from oracle import exact_topk

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "cuda-vector-search_b200" / "cuda_vector_search" / "libcvs_b200.so"
CVS_ERR_DEVICE_TIMEOUT = 5
ERR_TIMEOUT = 0x100
LOG_WAIT_SITES = {6, 7}  # iteration-log waits of the MMA issuer and of the drain warps


def _lib():
    lib = ctypes.CDLL(str(LIB))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.cvs_fused_topk.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, vp, ctypes.c_size_t, i32, i32, vp, vp]
    lib.cvs_fused_topk.restype = i32
    lib.cvs_fused_topk_workspace_size.argtypes = [i64, i64, i32, i32, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
    lib.cvs_fused_topk_workspace_size.restype = i32
    lib.cvs_debug_stall_next_search.argtypes = [i64]
    lib.cvs_debug_stall_next_search.restype = i32
    lib.cvs_poll_device_error.argtypes = [i32, ctypes.POINTER(ctypes.c_int)]
    lib.cvs_poll_device_error.restype = i32
    lib.cvs_last_error.restype = ctypes.c_char_p
    return lib


def _search(lib, q, x, k):
    b, n, d_pad = q.shape[0], x.shape[0], x.shape[1]
    nbytes = ctypes.c_size_t(0)
    assert lib.cvs_fused_topk_workspace_size(b, n, d_pad, k, 0, 0, ctypes.byref(nbytes)) == 0
    ws = torch.zeros(max(256, nbytes.value), dtype=torch.uint8, device=q.device)
    v = torch.empty((b, k), dtype=torch.float32, device=q.device)
    i = torch.empty((b, k), dtype=torch.int64, device=q.device)
    st = lib.cvs_fused_topk(q.data_ptr(), b, x.data_ptr(), n, d_pad, k, 0, v.data_ptr(), i.data_ptr(), ws.data_ptr(),
                            ws.numel(), 0, 0, None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return st, v.cpu(), i.cpu()


def _poll(lib):
    code = ctypes.c_int(-1)
    st = lib.cvs_poll_device_error(torch.cuda.current_device(), ctypes.byref(code))
    return st, code.value


@pytest.mark.parametrize("d", [512, 256])  # streamed and shared-memory-resident query tiles
def test_a_wait_that_runs_out_is_reported_and_the_gpu_stays_usable(d):
    lib = _lib()
    assert _poll(lib) == (0, 0), "an earlier kernel left an error behind"
    x, q = make(4000, d, 16, seed=d)  # past the GEMV's batches: the one-CTA tcgen05 kernel
    x, q = x.cuda(), q.cuda()
    assert lib.cvs_debug_stall_next_search(1_000_000) == 0
    st, _, _ = _search(lib, q, x, 10)
    assert st == 0, lib.cvs_last_error()  # the launch itself is fine; the kernel gives up on the device
    st, code = _poll(lib)
    assert st == CVS_ERR_DEVICE_TIMEOUT, lib.cvs_last_error()
    assert code & ERR_TIMEOUT and (code & 0xFF) in LOG_WAIT_SITES | {2}, hex(code)
    assert _poll(lib) == (0, 0)  # the poll cleared the word
    # The hook was one-shot: the same search now runs normally and is exact.
    st, v, i = _search(lib, q, x, 10)
    assert st == 0, lib.cvs_last_error()
    x32, q32 = x.float().cpu().numpy(), q.float().cpu().numpy()
    ref_v, ref_i = exact_topk(q32, x32, 11)
    assert_topk_exact(v.numpy(), i.numpy(), q32, x32, ref_v, ref_i, 10)
    assert _poll(lib) == (0, 0)


def test_the_hook_refuses_plans_it_does_not_cover():
    lib = _lib()
    x, q = make(3000, 128, 1, seed=1)  # one query, k <= 32: the GEMV plan
    x, q = x.cuda(), q.cuda()
    assert lib.cvs_debug_stall_next_search(1_000_000) == 0
    st, _, _ = _search(lib, q, x, 10)
    assert st == 1 and b"one-CTA" in lib.cvs_last_error()
    st, v, i = _search(lib, q, x, 10)  # disarmed
    assert st == 0
    assert lib.cvs_debug_stall_next_search(10) == 1  # limit out of range
    assert np.isfinite(v.numpy()).all()
    assert _poll(lib) == (0, 0)
