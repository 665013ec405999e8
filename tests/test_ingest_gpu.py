"""GPU ingest (dtype conversion + cosine normalisation + width padding) against
the oracle's restatement of the reference's _normalize_ / _pad_width
(cuda_vector_search/index.py:27-41): at most one fp16 ulp per element, almost
all elements bit-identical (the norm's summation order differs from torch's),
pad columns exactly zero. Covers the vectorised path (width % 8 == 0) and the
scalar path, every source dtype, and in-place use."""

import numpy as np
import pytest
import torch

from oracle import normalize_rows_fp16, pad_width

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mod():
    from cuda_vector_search import _ext

    assert _ext.available()
    return _ext.load()


def _ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(a.view(np.int16).astype(np.int32) - b.view(np.int16).astype(np.int32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("d", [64, 100, 384, 768, 1000, 1536, 2048])
@pytest.mark.parametrize("cosine", [True, False])
def test_ingest_matches_oracle(mod, dtype, d, cosine):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(1037, d, generator=g) * torch.rand(1037, 1, generator=g) * 3).to(dtype)
    d_pad = -(-d // 64) * 64
    out = torch.empty(1037, d_pad, dtype=torch.float16, device="cuda")
    mod.ingest_into(x.cuda(), out, cosine)
    got = out.cpu().numpy()
    src16 = x.to(torch.float16).numpy() if dtype != torch.float64 else x.numpy().astype(np.float16)
    ref = pad_width(normalize_rows_fp16(src16) if cosine else src16)
    u = _ulps(got, ref)
    assert u.max() <= 1
    assert (u == 0).mean() > 0.999
    assert not got[:, d:].any()


def test_ingest_in_place(mod):
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(3000, 512, generator=g) * 7).half()
    ref = normalize_rows_fp16(x.numpy())
    xd = x.cuda()
    mod.ingest_into(xd, xd, True)
    assert _ulps(xd.cpu().numpy(), ref).max() <= 1


def test_ingest_zero_rows_stay_finite(mod):
    x = torch.zeros(5, 128, device="cuda", dtype=torch.float32)
    out = torch.empty(5, 128, dtype=torch.float16, device="cuda")
    mod.ingest_into(x, out, True)
    assert torch.isfinite(out.float()).all() and not out.float().any()
