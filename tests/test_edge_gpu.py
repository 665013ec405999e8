"""GPU edge cases beyond the reference suite: every kernel variant (GEMV, one-CTA
tcgen05, CTA-pair tcgen05; register and buffer top-k; resident and streamed
queries), ragged tails, tiny corpora, k == n, exact ties, and the score kernel
on both tcgen05 variants. All compared with the CPU oracle on the stored rows."""

import numpy as np
import pytest
import torch

from helpers import assert_topk_exact
from oracle import exact_topk

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cvs():
    import cuda_vector_search as c
    from cuda_vector_search import _ext

    assert _ext.available(), "these tests need a B200 (sm_100) GPU"
    _ext.load()
    return c


def _data(n, d, b, seed, dup=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    x = x / x.norm(dim=1, keepdim=True)
    if dup:  # exact duplicate rows -> exact score ties
        x[dup::3] = x[0:len(x[dup::3])]
    q = torch.randn(b, d, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    return x.half(), q.half()


def _check(cvs, x, q, k, metric="ip", method="fused", chunks=None):
    index = cvs.Index(x.cuda(), metric=metric)
    if chunks is None:
        v, i = index.search(q.cuda(), k, method=method)
    else:
        from cuda_vector_search import _ext

        qq = index._prep_queries(q.cuda())
        v, i, _ = _ext.load().fused_topk(qq, index._x, k, 0, chunks)
    x32 = index.embeddings.float().cpu().numpy()
    q32 = index._prep_queries(q.cuda())[:, : index.dim].float().cpu().numpy()
    kk = min(k, x.shape[0])
    ref_v, ref_i = exact_topk(q32, x32, min(kk + 1, x.shape[0]))
    assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ref_v, ref_i, kk)
    return index, v, i


@pytest.mark.parametrize("b", [1, 2, 4, 5, 8, 9, 64, 127, 128, 129, 200, 256, 257, 384, 512])
def test_batch_sizes_across_kernel_boundaries(cvs, b):
    x, q = _data(6000, 384, b, seed=b)
    _check(cvs, x, q, 10)


@pytest.mark.parametrize("k", [1, 2, 15, 16, 17, 31, 32, 33, 64, 100, 255, 256, 512, 1024])
@pytest.mark.parametrize("b", [3, 100, 300])
def test_k_sweep(cvs, k, b):
    x, q = _data(5000, 192, b, seed=k * 7 + b)
    _check(cvs, x, q, k)


@pytest.mark.parametrize("d", [64, 128, 384, 448, 512, 768, 1024, 1536])
@pytest.mark.parametrize("b", [1, 50, 256])
def test_widths(cvs, d, b):
    x, q = _data(3000, d, b, seed=d + b)
    _check(cvs, x, q, 10)


@pytest.mark.parametrize("n", [1, 7, 255, 256, 257, 511, 513, 1000])
@pytest.mark.parametrize("b", [1, 20, 200])
def test_tiny_and_ragged_corpora(cvs, n, b):
    x, q = _data(n, 64, b, seed=n * 3 + b)
    _check(cvs, x, q, min(10, n))


@pytest.mark.parametrize("b", [2, 60, 160])
def test_k_equals_n(cvs, b):
    x, q = _data(300, 128, b, seed=b)
    _check(cvs, x, q, 300)


@pytest.mark.parametrize("b,k", [(1, 10), (3, 32), (40, 10), (40, 100), (200, 10), (200, 64)])
def test_exact_ties_choose_smaller_ids(cvs, b, k):
    """Rows 1, 4, 7, ... and 2, 5, 8, ... duplicate earlier rows: equal scores must
    come back smallest id first, and the kept set must be the oracle's."""
    x, q = _data(4000, 128, b, seed=99 + b, dup=1)
    index, v, i = _check(cvs, x, q, k)
    v, i = v.cpu().numpy(), i.cpu().numpy()
    for r in range(b):
        same = v[r, :-1] == v[r, 1:]
        assert (i[r, :-1][same] < i[r, 1:][same]).all()


@pytest.mark.parametrize("chunks", [1, 2, 3, 50, 10000])
@pytest.mark.parametrize("b,k", [(1, 10), (60, 10), (60, 64), (300, 10), (300, 100)])
def test_chunk_overrides(cvs, chunks, b, k):
    x, q = _data(9000, 256, b, seed=chunks + b + k)
    _check(cvs, x, q, k, chunks=chunks)


@pytest.mark.parametrize("b", [37, 129, 300])
def test_scores_both_tcgen05_variants(cvs, b):
    x, q = _data(3001, 192, b, seed=b)
    index = cvs.Index(x.cuda(), metric="ip")
    ref = q.float() @ x.float().T
    s = index.scores(q.cuda())
    assert s.shape == (b, 3001)
    assert torch.allclose(s.cpu(), ref, atol=1e-3)
    s16 = index.scores(q.cuda(), fp32=False)
    assert torch.allclose(s16.float().cpu(), ref, atol=3e-3)


def test_cosine_large_batch_pair_path(cvs):
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(20000, 768, generator=g) * torch.rand(20000, 1, generator=g) * 5).half()
    q = torch.randn(300, 768, generator=g).half()
    _check(cvs, x, q, 10, metric="cosine")


def test_repeated_calls_are_deterministic(cvs):
    x, q = _data(30000, 768, 256, seed=3)
    index = cvs.Index(x.cuda(), metric="ip")
    a = index.search(q.cuda(), 10)
    for _ in range(3):
        b = index.search(q.cuda(), 10)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_no_device_errors_after_edges(cvs):
    from cuda_vector_search import _ext

    torch.cuda.synchronize()
    assert _ext.load().poll_device_error(torch.cuda.current_device()) == 0


# Dry tiles (each CTA reads its first one or two claimed tiles twice: once to
# publish bounds, once for real after its last tile); chunk overrides and a
# larger corpus force every regime: 1 tile per CTA (its only tile read dry
# first), 2 (one dry tile), 3 and more (two). b = 1 and, on the small corpus,
# b = 3 run on the GEMV instead.
@pytest.mark.parametrize("chunks", [0, 3, 8, 30, 60])
@pytest.mark.parametrize("b,k", [(1, 10), (3, 10), (70, 10), (70, 24), (70, 64), (300, 10), (300, 200)])
def test_dry_tile_regimes(cvs, chunks, b, k):
    x, q = _data(120000 if chunks == 0 else 15360, 128, b, seed=chunks * 31 + b + k)
    _check(cvs, x, q, k, chunks=chunks if chunks else None)


# The GEMV takes one query at every corpus size, and two to eight queries on
# corpora of at most two tiles per CTA (5000 rows: 20 tiles; 60000: 235; 148
# SMs) with resident-width query tiles (d_pad <= 640) while rows x
# max(d_pad, 256) x the instantiation's queries stays below 3e7 (k = 10).
# 120000 rows is 469 tiles.
@pytest.mark.parametrize("n,d,b,expect_gemv", [(5000, 256, 1, True), (5000, 256, 2, True), (5000, 256, 3, True),
                                               (5000, 256, 4, True), (5000, 256, 5, True), (5000, 256, 8, True),
                                               (5000, 256, 9, False), (12000, 256, 8, True), (12000, 128, 8, True),
                                               (60000, 256, 2, False), (60000, 256, 8, False),
                                               (30000, 1024, 4, False), (120000, 256, 1, True),
                                               (120000, 256, 2, False), (120000, 256, 8, False)])
def test_plan_selects_gemv(cvs, n, d, b, expect_gemv):
    from cuda_vector_search import _ext

    x, q = _data(n, d, b, seed=b)
    index = cvs.Index(x.cuda(), metric="ip")
    v, i, plan = _ext.load().fused_topk(index._prep_queries(q.cuda()), index._x, 10)
    assert (plan.tolist()[0] == b) == expect_gemv  # GEMV plans echo b, tcgen05 plans the tile
    v2, i2, plan2 = _ext.load().fused_topk(index._prep_queries(q.cuda()), index._x, 10, 64)
    assert plan2.tolist()[0] == 64  # an explicit bq always selects tcgen05 tiles
    assert torch.equal(i, i2)


# The GEMV's 2-, 4- and 8-query instantiations against the oracle (padded
# query slots of a 3-, 5-, 6- or 7-query batch included), with duplicated rows
# for exact ties and a ragged width, on plans asserted to be GEMV plans.
@pytest.mark.parametrize("n,d,b,k,dup", [(3000, 100, 2, 10, 0), (20011, 384, 3, 17, 0), (9000, 640, 4, 32, 1),
                                         (5000, 256, 5, 10, 2), (12345, 384, 6, 32, 0), (1000, 64, 7, 1, 1),
                                         (20000, 128, 8, 32, 0), (40, 256, 8, 32, 1)])
def test_gemv_batches_match_oracle(cvs, n, d, b, k, dup):
    from cuda_vector_search import _ext

    x, q = _data(n, d, b, seed=n + b, dup=dup)
    index, v, i = _check(cvs, x, q, k)
    _, _, plan = _ext.load().fused_topk(index._prep_queries(q.cuda()), index._x, k)
    assert plan.tolist()[0] == b  # the GEMV plan


def test_pinned_host_queries_back_to_back(cvs):
    """Pinned host query blocks of 256 KB and more go through a ring of four
    device upload slots on a side stream. Ten searches issued back to back behind
    a busy stream (no host synchronisation between them) must each see their own
    queries: a slot is refilled only after the ingest that read it has run, and a
    slot that grows, or changes dtype, keeps its old buffer alive for queued work."""
    import cuda_vector_search.index as ix

    x, q = _data(20000, 256, 3600, seed=5)
    index = cvs.Index(x.cuda(), metric="cosine")
    sizes = [260, 300, 280, 320, 400, 260, 300, 500, 270, 290]  # rows of 256 fp32 >= 256 KB
    starts = [sum(sizes[:j]) for j in range(len(sizes))]
    parts = [q[s0:s0 + n].float() for s0, n in zip(starts, sizes)]
    parts[6] = parts[6].double()  # a slot switching dtype
    ref = [index.search(p.cuda(), 10) for p in parts]
    pinned = [p.pin_memory() for p in parts]
    assert all(p.nbytes >= ix._SIDE_UPLOAD_BYTES for p in pinned)
    torch.cuda.synchronize()
    torch.cuda._sleep(20_000_000)  # the host runs ahead of the GPU
    outs = [index.search(p, 10) for p in pinned]
    torch.cuda.synchronize()
    for (rv, ri), (v, i) in zip(ref, outs):
        assert torch.equal(ri, i)
        assert torch.equal(rv, v)


@pytest.mark.parametrize("b,tile", [(200, 256), (256, 256), (300, 128), (384, 128), (512, 256), (640, 128)])
def test_plan_prefers_the_tile_with_fewer_padded_rows(cvs, b, tile):
    """CTA pairs (256-query tiles) unless 128-query tiles pad fewer rows; results
    are the oracle's either way."""
    from cuda_vector_search import _ext

    x, q = _data(6000, 128, b, seed=b + 7)
    index = cvs.Index(x.cuda(), metric="ip")
    v, i, plan = _ext.load().fused_topk(index._prep_queries(q.cuda()), index._x, 10)
    assert plan.tolist()[0] == tile
    _check(cvs, x, q, 10)
