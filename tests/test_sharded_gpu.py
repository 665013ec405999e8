"""Sharded search on the GPU.

* Simulated on one GPU: the corpus is split into S pseudo-shards, each searched
  with its global row offset (fused_topk_into), the [S, b, k] lists merged with
  merge_lists; the result must match the CPU oracle on the global corpus and
  equal the unsharded search exactly.
* Real ranks: when at least two GPUs are visible, tests/mp_sharded_check.py runs
  under torchrun with NCCL and compares ShardedIndex with the CPU oracle on the
  global corpus and with a single-GPU Index.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from helpers import assert_topk_exact
from oracle import exact_topk

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def mod():
    from cuda_vector_search import _ext

    assert _ext.available()
    return _ext.load()


@pytest.mark.parametrize("n,d,b,k,shards", [(20000, 384, 64, 10, 4), (20000, 768, 300, 32, 3),
                                            (9000, 128, 5, 100, 7), (5000, 256, 1, 10, 2)])
def test_simulated_sharding_equals_unsharded(mod, n, d, b, k, shards):
    import cuda_vector_search as cvs

    g = torch.Generator().manual_seed(n + b)
    x = torch.randn(n, d, generator=g).half().cuda()
    q = torch.randn(b, d, generator=g).half().cuda()
    full = cvs.Index(x, metric="cosine")
    ref_v, ref_i = full.search(q, k)
    bounds = [round(s * n / shards) for s in range(shards + 1)]
    vs, ids = [], []
    for s in range(shards):
        part = cvs.Index(x[bounds[s]:bounds[s + 1]], metric="cosine")
        qq = part._prep_queries(q)
        kk = min(k, len(part))
        v = torch.empty(b, kk, device="cuda")
        i = torch.empty(b, kk, dtype=torch.int64, device="cuda")
        ws = torch.empty(max(256, mod.workspace_size(b, len(part), part._x.shape[1], kk)), dtype=torch.uint8,
                         device="cuda")
        mod.fused_topk_into(qq, part._x, kk, bounds[s], v, i, ws)
        if kk < k:
            v = torch.cat([v, v.new_full((b, k - kk), float("-inf"))], 1)
            i = torch.cat([i, i.new_full((b, k - kk), -1)], 1)
        vs.append(v)
        ids.append(i)
    mv, mi = mod.merge_lists(torch.stack(vs).contiguous(), torch.stack(ids).contiguous(), k)
    # Against the CPU oracle on the stored (normalised) global corpus ...
    x32 = full.embeddings.float().cpu().numpy()
    q32 = full._prep_queries(q)[:, :d].float().cpu().numpy()
    ov, oi = exact_topk(q32, x32, min(k + 1, n))
    assert_topk_exact(mv.cpu().numpy(), mi.cpu().numpy(), q32, x32, ov, oi, k)
    # ... and bit for bit against the unsharded search.
    assert torch.equal(mi, ref_i)
    assert torch.allclose(mv, ref_v, atol=1e-6, rtol=0)


def test_nccl_ranks_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT), str(ROOT / "cuda-vector-search_b200"),
                                                        os.environ.get("PYTHONPATH", "")]))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           str(ROOT / "tests" / "mp_sharded_check.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=360)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "SHARDED OK" in res.stdout


def test_save_then_load_whole_and_per_shard_ranges(mod, tmp_path):
    """Index.save, then (a) Index.load, which maps the .npy and stages it in
    chunks, and (b) the per-rank row ranges ShardedIndex.load ingests
    (load_shard_rows), searched as pseudo-shards on this GPU and merged: both
    match the CPU oracle on the saved corpus."""
    import numpy as np

    import cuda_vector_search as cvs
    from cuda_vector_search.sharded import load_shard_rows

    g = torch.Generator().manual_seed(11)
    n, d, b, k, shards = 300_001, 200, 40, 25, 3  # > one 2^18-row staging chunk, ragged ranges
    x = torch.randn(n, d, generator=g).half()
    q = torch.randn(b, d, generator=g).half().cuda()
    path = tmp_path / "corpus.npy"
    cvs.Index(x.cuda(), metric="cosine").save(path)
    saved = np.load(path)
    whole = cvs.Index.load(path)
    assert whole.metric == "cosine" and len(whole) == n and whole.dim == d
    q32 = whole._prep_queries(q)[:, :d].float().cpu().numpy()
    x32 = whole.embeddings.float().cpu().numpy()
    ov, oi = exact_topk(q32, x32, k + 1)
    v, i = whole.search(q, k)
    assert_topk_exact(v.cpu().numpy(), i.cpu().numpy(), q32, x32, ov, oi, k)
    vs, ids = [], []
    for r in range(shards):
        rows, lo, metric = load_shard_rows(path, r, shards)
        assert lo == n * r // shards and metric == "cosine"
        assert np.array_equal(np.asarray(rows), saved[lo:lo + rows.shape[0]])
        part = cvs.Index(rows, metric=metric)
        pv = torch.empty(b, k, device="cuda")
        pi = torch.empty(b, k, dtype=torch.int64, device="cuda")
        ws = torch.empty(max(256, mod.workspace_size(b, len(part), part._x.shape[1], k)), dtype=torch.uint8,
                         device="cuda")
        mod.fused_topk_into(part._prep_queries(q), part._x, k, lo, pv, pi, ws)
        vs.append(pv)
        ids.append(pi)
    mv, mi = mod.merge_lists(torch.stack(vs).contiguous(), torch.stack(ids).contiguous(), k)
    assert_topk_exact(mv.cpu().numpy(), mi.cpu().numpy(), q32, x32, ov, oi, k)


@pytest.mark.parametrize("lists,b,length,k", [(8, 256, 10, 10), (8, 300, 100, 100), (5, 64, 256, 200),
                                              (3, 40, 1024, 1024), (2, 7, 17, 5)])
def test_merge_lists_matches_the_oracle_merge(mod, lists, b, length, k):
    """merge_lists (the merge after the all-gather) against oracle.merge_topk,
    with exact score ties across lists and empty slots (id -1) in short shards;
    the first four shapes take the shared-memory staged path, (3, 40, 1024)
    the global-memory one."""
    import numpy as np

    from oracle import merge_topk

    g = torch.Generator().manual_seed(lists * 1000 + length)
    v = torch.randn(lists, b, length, generator=g).round(decimals=2)  # many exact ties
    ids = torch.stack([torch.stack([torch.randperm(1 << 20, generator=g)[:length] + (l << 20) for _ in range(b)])
                       for l in range(lists)])
    v, order = v.sort(dim=2, descending=True)
    ids = ids.gather(2, order)
    ids[0, :, length - 3:] = -1  # a shard with fewer rows than k: empty slots
    v[0, :, length - 3:] = float("-inf")
    mv, mi = mod.merge_lists(v.cuda().contiguous(), ids.cuda().contiguous(), k)
    vs = [np.where(ids[l].numpy() >= 0, v[l].numpy(), -np.inf).astype(np.float32) for l in range(lists)]
    js = [np.where(ids[l].numpy() >= 0, ids[l].numpy(), np.iinfo(np.int64).max) for l in range(lists)]
    rv, ri = merge_topk(vs, js, k)
    ri = np.where(ri == np.iinfo(np.int64).max, -1, ri)
    assert np.array_equal(mi.cpu().numpy(), ri)
    assert np.array_equal(mv.cpu().numpy(), rv)
