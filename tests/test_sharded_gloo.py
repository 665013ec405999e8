"""Row-sharded search across ranks (ShardedIndex), run as world-size-2 `gloo`
process groups on the CPU. The per-rank search and the merge are the CPU oracle
injected through ShardOps, so what is tested here is the host logic the GPU
path shares: shard sizes and global row offsets, padding of shards smaller
than k, the all-gather layout, the exact global order after the merge, and how
a rank failure surfaces (a collective with a short timeout raises instead of
hanging). The reference has no multi-GPU path; its chunked ground truth
(cuda_vector_search/reference.py:22-33) is the template being distributed."""

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

from oracle import exact_topk, merge_topk


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _corpus(n=3000, d=48, b=5, seed=0, dup=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, d)).astype(np.float16)
    if dup:
        x[1::2] = x[0::2][: len(x[1::2])]  # exact ties across shard boundaries
    q = rng.standard_normal((b, d)).astype(np.float16)
    return x, q


def _cpu_ops(shard: np.ndarray):
    from cuda_vector_search.sharded import ShardOps

    def local_topk(queries, k, id_offset):
        q = np.asarray(queries, dtype=np.float32)
        kk = min(k, shard.shape[0])
        v, i = exact_topk(q, shard, kk)
        v = torch.from_numpy(v)
        i = torch.from_numpy(i + id_offset)
        if kk < k:
            v = torch.cat([v, v.new_full((v.shape[0], k - kk), float("-inf"))], 1)
            i = torch.cat([i, i.new_full((i.shape[0], k - kk), -1)], 1)
        return v, i

    def merge(v_all, i_all, k):
        vs = [v_all[r].numpy() for r in range(v_all.shape[0])]
        ids = [i_all[r].numpy() for r in range(i_all.shape[0])]
        # empty slots (-1) rank last
        vs = [np.where(i >= 0, v, -np.inf).astype(np.float32) for v, i in zip(vs, ids)]
        ids = [np.where(i >= 0, i, np.iinfo(np.int64).max) for i in ids]
        v, i = merge_topk(vs, ids, k)
        return torch.from_numpy(v), torch.from_numpy(i)

    return ShardOps(local_topk=local_topk, merge=merge, n_local=shard.shape[0], device=torch.device("cpu"))


def _worker(rank, world, port, case, out):
    try:
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parent.parent
        sys.path[:0] = [str(root), str(root / "cuda-vector-search_b200"), str(root / "tests")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        from cuda_vector_search import ShardedIndex

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=case.get("timeout", 60)))
        x, q = _corpus(**case["data"])
        if case.get("load"):
            # Each rank maps the saved file and takes only its own row range.
            idx = ShardedIndex.load(case["load"], ops_factory=lambda rows: _cpu_ops(np.asarray(rows)))
        else:
            bounds = case["bounds"]
            shard = x[bounds[rank]:bounds[rank + 1]]
            idx = ShardedIndex(ops=_cpu_ops(shard))
        if case.get("fail_rank") == rank:
            raise SystemExit(3)  # this rank leaves before the collective search
        v, i = idx.search(q.astype(np.float32), case["k"])
        out.put((rank, "ok", idx.row_offset, idx.n_total, v.numpy(), i.numpy()))
        dist.destroy_process_group()
    except SystemExit:
        out.put((rank, "exited", None, None, None, None))
    except Exception:
        out.put((rank, "error", traceback.format_exc(), None, None, None))


def _run(case, world=2):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return {r[0]: r[1:] for r in res}


@pytest.mark.parametrize("bounds,k", [((0, 1500, 3000), 10), ((0, 7, 3000), 10), ((0, 2990, 3000), 25)])
def test_sharded_equals_unsharded(bounds, k):
    case = dict(data=dict(n=3000, d=48, b=5, seed=1), bounds=bounds, k=k)
    res = _run(case)
    x, q = _corpus(**case["data"])
    ref_v, ref_i = exact_topk(q.astype(np.float32), x, k)
    for rank in (0, 1):
        status, offset, total, v, i = res[rank]
        assert status == "ok", offset
        assert offset == bounds[rank] and total == 3000
        np.testing.assert_allclose(v, ref_v, rtol=0, atol=1e-5)
        assert (i == ref_i).all()


def test_sharded_ties_keep_global_id_order():
    case = dict(data=dict(n=2000, d=32, b=4, seed=2, dup=True), bounds=(0, 1001, 2000), k=12)
    res = _run(case)
    x, q = _corpus(**case["data"])
    ref_v, ref_i = exact_topk(q.astype(np.float32), x, 12)
    status, _, _, v, i = res[0]
    assert status == "ok"
    assert (i == ref_i).all()


def test_a_rank_that_leaves_makes_the_others_fail_not_hang():
    case = dict(data=dict(n=1000, d=16, b=2, seed=3), bounds=(0, 500, 1000), k=5, fail_rank=1, timeout=5)
    res = _run(case)
    assert res[1][0] == "exited"
    assert res[0][0] == "error"  # the collective search raised after the short timeout


def test_sharded_load_maps_each_ranks_row_range(tmp_path):
    """ShardedIndex.load: rank r of W ingests rows [n*r//W, n*(r+1)//W) of one
    saved .npy (the format Index.save writes); the global result equals the
    oracle on the whole file."""
    data = dict(n=3001, d=48, b=5, seed=4)
    x, q = _corpus(**data)
    path = tmp_path / "corpus.npy"
    np.save(path, x)
    (tmp_path / "corpus.npy.json").write_text('{"metric": "ip", "dim": 48, "n": 3001}')
    res = _run(dict(data=data, load=str(path), k=17))
    ref_v, ref_i = exact_topk(q.astype(np.float32), x, 17)
    for rank, lo in ((0, 0), (1, 1500)):
        status, offset, total, v, i = res[rank]
        assert status == "ok", offset
        assert offset == lo and total == 3001
        np.testing.assert_allclose(v, ref_v, rtol=0, atol=1e-5)
        assert (i == ref_i).all()


def test_a_rank_without_rows_fails_on_every_rank():
    """An empty shard is reported by every rank at construction (after the one
    collective that gathers the shard sizes), not by a hang in a later search."""
    case = dict(data=dict(n=1000, d=16, b=2, seed=3), bounds=(0, 0, 1000), k=5, timeout=20)
    res = _run(case)
    for rank in (0, 1):
        assert res[rank][0] == "error"
        assert "at least one row" in res[rank][1]


def test_shape_cache_keeps_only_recent_shapes():
    """The per-(batch, k) buffers of the sharded path are bounded (LRU)."""
    from collections import OrderedDict

    from cuda_vector_search.sharded import _CACHED_SHAPES, _cached

    cache = OrderedDict()
    made = []
    for key in [(1, 10), (2, 10), (1, 10), (3, 10), (4, 10), (5, 10), (1, 10)]:
        _cached(cache, key, lambda key=key: made.append(key) or key)
    assert len(cache) == _CACHED_SHAPES
    assert list(cache)[-1] == (1, 10)
    assert made.count((1, 10)) == 1 and (2, 10) not in cache
