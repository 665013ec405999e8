"""Host-side behaviour that needs no GPU: the product refuses to run without an
sm_100 device (no CPU fallback), the torch binding enforces the reference's
input contract (cuda_vector_search/csrc/kernels.cu:451-470), and the API
validation mirrors the reference's (cuda_vector_search/index.py:57-63, 110-115)."""

import numpy as np
import pytest
import torch

import cuda_vector_search as cvs
from cuda_vector_search import _C, _ext


def test_package_exports_the_reference_api():
    for name in ("Index", "exact_topk_fp32", "torch_topk", "ShardedIndex", "__version__"):
        assert hasattr(cvs, name)


def test_no_cpu_fallback():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert not _ext.available()
    with pytest.raises(RuntimeError):
        _ext.load()
    with pytest.raises(RuntimeError):
        cvs.Index(np.ones((10, 8), np.float32))
    with pytest.raises(RuntimeError):
        cvs.Index(np.ones((10, 8), np.float32), device="cpu")


def test_index_argument_validation_precedes_device_checks():
    with pytest.raises(ValueError):
        cvs.Index(np.ones((10, 8), np.float32), metric="l2")
    with pytest.raises(ValueError):
        cvs.Index(np.ones(8, np.float32))
    with pytest.raises(ValueError):
        cvs.Index(np.ones((0, 8), np.float32))


def test_binding_rejects_non_cuda_inputs_like_the_reference():
    q = torch.zeros(4, 64, dtype=torch.float16)
    x = torch.zeros(100, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _C.fused_topk(q, x, 10, 0, 0)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _C.scores(q, x, True)


def test_exact_topk_fp32_helper_on_cpu():
    """The exported ground-truth helper (reference.py:18-34) behaves the same on CPU."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5000, 32, generator=g)
    q = torch.randn(3, 32, generator=g)
    v, i = cvs.exact_topk_fp32(q, x, 7, chunk=333)
    rv, ri = torch.topk(q @ x.T, 7, dim=1)
    assert torch.allclose(v, rv, atol=1e-5) and torch.equal(i, ri)
