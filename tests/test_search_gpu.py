"""GPU parity: the reference's test suite (tests/test_search.py of
sonhoang/cuda-vector-search) run against this build, with every case checked
twice -- against the CPU oracle on this index's own stored vectors, and against
the golden vectors the reference itself produced."""

import numpy as np
import pytest
import torch

from cases import BY_NAME, FUSED, make
from helpers import assert_topk_exact, golden, true_scores
from oracle import exact_topk

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cvs():
    import cuda_vector_search as c
    from cuda_vector_search import _ext

    assert _ext.available(), "these tests need a B200 (sm_100) GPU"
    _ext.load()
    return c


def stored(index) -> np.ndarray:
    return index.embeddings.float().cpu().numpy()


def prepped(index, q) -> np.ndarray:
    return index._prep_queries(q)[:, : index.dim].float().cpu().numpy()


def build(cvs, name):
    c = BY_NAME[name]
    x, q = make(c["n"], c["d"], c["b"], seed=c["seed"], normal=c["normal"],
                scale_rows=c.get("scale_rows", False))
    index = cvs.Index(x.cuda(), metric=c["metric"])
    return c, index, q.cuda()


def check_case(cvs, name, method="fused", k=None):
    c, index, q = build(cvs, name)
    k = min(k or c["k"], c["n"])
    v, i = index.search(q, k, method=method)
    torch.cuda.synchronize()
    assert v.dtype == torch.float32 and i.dtype == torch.int64
    assert v.device == index.device and i.device == index.device
    x32, q32 = stored(index), prepped(index, q)
    ref_v, ref_i = exact_topk(q32, x32, min(k + 1, c["n"]))
    scale = max(1.0, float(np.abs(ref_v).max()))
    assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ref_v, ref_i, k, scale=scale)
    _, gv, gi = golden(name)
    rel = 1e-5 if c["metric"] == "ip" else 1e-4  # see test_oracle: cosine rows may differ by 1 ulp
    if k <= gv.shape[1]:
        assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, gv, gi, k, rel=rel, scale=scale)
    return index, q, v, i


@pytest.mark.parametrize("n,d,b,k", FUSED)
def test_fused_matches_exact(cvs, n, d, b, k):
    check_case(cvs, f"fused_{n}_{d}_{b}_{k}", method="fused")


@pytest.mark.parametrize("name", ["gemv_1_768_10", "gemv_2_768_32", "gemv_3_384_17", "gemv_5_1024_10",
                                  "gemv_8_768_32", "cosine_pad_100", "ragged_129_1000", "wide_1536"])
def test_added_cases(cvs, name):
    check_case(cvs, name, method="auto")


@pytest.mark.parametrize("name", ["twopass_5000_384_8_10", "twopass_20000_768_64_100"])
def test_twopass_and_torch_paths(cvs, name):
    """These paths keep fp16 scores: the reference contract with tol 2e-3 (test_search.py:72-80)."""
    c, index, q = build(cvs, name)
    x32, q32 = stored(index), prepped(index, q)
    ref_v, _ = exact_topk(q32, x32, c["k"])
    for method in ("twopass", "torch"):
        v, i = index.search(q, c["k"], method=method)
        v, i = v.cpu().numpy(), i.cpu().numpy()
        ts = true_scores(q32, x32, i)
        assert np.abs(v - ts).max() <= 2e-3
        assert (ts >= ref_v[:, -1:] - 2e-3).all()
        assert (v[:, :-1] >= v[:, 1:] - 1e-6).all()
        for row in i:
            assert len(set(row.tolist())) == c["k"]


def test_cosine_metric_unnormalised_input(cvs):
    """test_search.py:83-92: varied row norms, cosine metric, vs fp32 cosine on CPU."""
    index, q, v, i = check_case(cvs, "cosine_unnormalised", method="auto")
    c = BY_NAME["cosine_unnormalised"]
    x, qh = make(c["n"], c["d"], c["b"], seed=c["seed"], normal=False, scale_rows=True)
    xn = x.float() / x.float().norm(dim=1, keepdim=True)
    qn = qh.float() / qh.float().norm(dim=1, keepdim=True)
    ref_v, _ = torch.topk(qn @ xn.T, 10, dim=1)
    assert torch.allclose(v.cpu(), ref_v, atol=3e-3)


def test_raw_ip_large_values(cvs):
    """test_search.py:95-100: unnormalised inner products (|s| ~ 16-60)."""
    check_case(cvs, "raw_ip_large", method="fused")


def test_scores_kernel_matches_fp32(cvs):
    """test_search.py:103-113."""
    c, index, q = build(cvs, "scores_3001_192_37")
    x, qh = make(c["n"], c["d"], c["b"], seed=c["seed"])
    s = index.scores(q)
    ref = qh.float() @ x.float().T
    assert s.shape == (37, 3001) and s.dtype == torch.float32
    assert torch.allclose(s.cpu(), ref, atol=1e-3)
    s16 = index.scores(q, fp32=False)
    assert s16.dtype == torch.float16
    assert torch.allclose(s16.float().cpu(), ref, atol=3e-3)


def test_exact_reference_helper(cvs):
    """test_search.py:116-121: the exported fp32 helper, on the GPU."""
    x, q = make(70000, 128, 4, seed=9)
    v, i = cvs.exact_topk_fp32(q.cuda(), x.cuda(), 20, chunk=8192)
    ref_v, _ = torch.topk(q.float() @ x.float().T, 20, dim=1)
    assert torch.allclose(v.cpu(), ref_v, atol=1e-5)


def test_one_dim_query_and_large_k(cvs):
    """test_search.py:124-131; k=400 now runs on the fused kernels (limit 1024 here)."""
    x, q = make(5000, 128, 1, seed=2)
    index = cvs.Index(x.cuda(), metric="ip")
    v, i = index.search(q[0].cuda(), 5)
    assert v.shape == (1, 5)
    v, i = index.search(q.cuda(), 400)
    assert i.shape == (1, 400)
    x32, q32 = stored(index), prepped(index, q.cuda())
    ref_v, ref_i = exact_topk(q32, x32, 401)
    assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ref_v, ref_i, 400)
    v, i = index.search(q.cuda(), 1500)  # beyond the fused limit -> twopass
    assert i.shape == (1, 1500)
    # twopass keeps fp16 scores: the reference contract at its 2e-3 tolerance
    # (test_search.py:72-80), against the fp32 oracle.
    ref_v, _ = exact_topk(q32, x32, 1500)
    v, i = v.cpu().numpy(), i.cpu().numpy()
    ts = true_scores(q32, x32, i)
    assert np.abs(v - ts).max() <= 2e-3
    assert (ts >= ref_v[:, -1:] - 2e-3).all()
    assert (v[:, :-1] >= v[:, 1:] - 1e-6).all()
    assert len(set(i[0].tolist())) == 1500


def test_fused_plan_overrides(cvs):
    """test_search.py:134-143: explicit bq / chunks give the same results; bq is echoed."""
    from cuda_vector_search import _ext

    mod = _ext.load()
    c, index, q = build(cvs, "plan_overrides")
    qq = index._prep_queries(q)
    x32, q32 = stored(index), prepped(index, q)
    ref_v, ref_i = exact_topk(q32, x32, 11)
    base_v, base_i = index.search(q, 10, method="fused")
    assert_topk_exact(base_v.cpu().numpy(), base_i.cpu().numpy(), q32, x32, ref_v, ref_i, 10)
    for bq, chunks in [(16, 1), (32, 7), (64, 1000), (256, 3)]:
        v, i, plan = mod.fused_topk(qq, index._x, 10, bq, chunks)
        assert plan.tolist()[0] == bq
        assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ref_v, ref_i, 10)
        assert torch.allclose(v, base_v, atol=1e-5)
        assert torch.equal(i, base_i)


def test_save_load_roundtrip(cvs, tmp_path):
    """test_search.py:146-156 (on the GPU: this build has no CPU index)."""
    x, q = make(500, 64, 3, seed=1, normal=False)
    index = cvs.Index(x.float().numpy(), metric="cosine")
    path = tmp_path / "emb.npy"
    index.save(path)
    again = cvs.Index.load(path)
    assert again.metric == "cosine" and len(again) == 500 and again.dim == 64
    a = index.search(q.float().numpy(), 5)
    b = again.search(q.float().numpy(), 5)
    assert torch.equal(a[1].cpu(), b[1].cpu())
    assert np.load(path).dtype == np.float16


@pytest.mark.parametrize("k,bq", [(100, 64), (256, 32), (200, 16), (40, 64)])
def test_fused_large_state_configs(cvs, k, bq):
    """test_search.py:159-168."""
    from cuda_vector_search import _ext

    mod = _ext.load()
    c, index, q = build(cvs, f"large_state_{k}_{bq}")
    qq = index._prep_queries(q)
    x32, q32 = stored(index), prepped(index, q)
    ref_v, ref_i = exact_topk(q32, x32, k + 1)
    for chunks in (1, 5, 0):
        v, i, plan = mod.fused_topk(qq, index._x, k, bq, chunks)
        assert plan.tolist()[0] == bq
        assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ref_v, ref_i, k)


def test_no_device_errors(cvs):
    """No kernel of the suite reported a failed pipeline wait."""
    from cuda_vector_search import _ext

    assert _ext.load().poll_device_error(torch.cuda.current_device()) == 0
