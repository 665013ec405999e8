"""cvs_search through the C ABI: raw queries of every supported dtype and a
row stride wider than the width, prepared (converted, normalised, padded) in
the search's first launch; results checked against the CPU oracle on the
queries prepared by the ingest entry point (the same arithmetic)."""

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
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


def _lib():
    lib = ctypes.CDLL(str(LIB))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.cvs_search.argtypes = [vp, i32, i64, i32, i64, i32, vp, i64, i32, i32, i64, vp, vp, vp, ctypes.c_size_t, vp]
    lib.cvs_search.restype = i32
    lib.cvs_search_workspace_size.argtypes = [i64, i64, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
    lib.cvs_search_workspace_size.restype = i32
    lib.cvs_ingest.argtypes = [vp, i32, i64, i32, i64, i32, i32, vp, vp]
    lib.cvs_ingest.restype = i32
    lib.cvs_last_error.restype = ctypes.c_char_p
    return lib


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("b,k,cosine", [(1, 10, 1), (7, 10, 1), (200, 100, 0), (129, 33, 1)])
def test_search_from_raw_strided_queries(dtype, b, k, cosine):
    lib = _lib()
    n, d = 30000, 300  # d_pad 320: padding columns are written by the preparation
    x, _ = make(n, d, 1, seed=b + k)
    d_pad = 320
    xs = torch.zeros(n, d_pad, dtype=torch.float16, device="cuda")
    xs[:, :d] = x.cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if cosine:  # stored rows normalised like the index does
        assert lib.cvs_ingest(xs.data_ptr(), 1, n, d_pad, d_pad, d_pad, 1, xs.data_ptr(), stream) == 0
    g = torch.Generator().manual_seed(b)
    wide = torch.randn(b, d + 17, generator=g).to(dtype).cuda()  # row stride d + 17 elements
    q = wide[:, :d]
    nbytes = ctypes.c_size_t(0)
    assert lib.cvs_search_workspace_size(b, n, d_pad, k, ctypes.byref(nbytes)) == 0
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    v = torch.empty(b, k, device="cuda")
    i = torch.empty(b, k, dtype=torch.int64, device="cuda")
    for _ in range(2):  # the second call starts from the first call's workspace contents
        st = lib.cvs_search(q.data_ptr(), DTYPES[dtype], b, d, q.stride(0), cosine, xs.data_ptr(), n, d_pad, k, 5,
                            v.data_ptr(), i.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        assert st == 0, lib.cvs_last_error()
        qp = torch.empty(b, d_pad, dtype=torch.float16, device="cuda")
        assert lib.cvs_ingest(q.data_ptr(), DTYPES[dtype], b, d, q.stride(0), d_pad, cosine, qp.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        x32 = xs[:, :d].float().cpu().numpy()
        q32 = qp[:, :d].float().cpu().numpy()
        ov, oi = exact_topk(q32, x32, k + 1)
        got_i = i.cpu().numpy() - 5  # id_offset
        scale = max(1.0, float(np.abs(ov).max()))
        assert_topk_exact(v.cpu().numpy(), got_i, q32, x32, ov, oi, k, scale=scale)
