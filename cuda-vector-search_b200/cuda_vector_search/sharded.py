"""Row-sharded exact search across GPUs: one process per GPU, torch.distributed.

The reference has no multi-GPU path; its chunked ground truth
(cuda_vector_search/reference.py:22-33: local top-k per chunk, ids shifted by the
chunk start, concatenate, top-k again) is the template. Here each rank owns a
contiguous row range of the corpus, runs the fused search on it with its global
row offset folded into the ids, the ranks all-gather their [b, k] (score, id)
lists (NCCL over NVLink), and every rank merges the [world, b, k] lists with the
merge kernel. There is exactly one collective per search: each rank's ids and
scores sit in one block (12 * b * k bytes, rounded up to 8), the search writes
them there directly, and the merge reads them straight out of the gathered
blocks.

Ordering is exact and global: score descending, then smaller global id, the same
rule as the single-GPU index, because every per-rank list is complete for its
rows and the merge compares (score, global id) keys.
"""

from __future__ import annotations

import json
from collections import OrderedDict
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import numpy as np
import torch
import torch.distributed as dist

from . import _ext
from .index import MAX_FUSED_K, Index, _to_tensor


def all_gather_stacked(t: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """[world, *t.shape] gather of ``t`` from every rank (same shape everywhere),
    into ``out`` when given."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


@dataclass
class ShardOps:
    """The per-rank operations a sharded search needs.

    local_topk(queries, k, id_offset) -> (scores [b, k] f32, ids [b, k] i64, sorted
    best first, ids already global, empty slots id -1); merge(scores [W, b, k],
    ids [W, b, k], k) -> (scores [b, k], ids [b, k]) (each [b, k] list dense, the W
    lists any stride apart). local_topk_into(queries, k, id_offset, scores_out,
    ids_out), if given, writes the local result into the given [b, k] tensors.
    """

    local_topk: Callable
    merge: Callable
    n_local: int
    device: torch.device
    local_topk_into: Callable | None = None


_CACHED_SHAPES = 4  # (batch, k) shapes whose buffers are kept for reuse


def _cached(cache: OrderedDict, key, make):
    """cache[key], created by make() on a miss; only the most recently used
    _CACHED_SHAPES entries are kept (a server with varying batch sizes must not
    accumulate workspaces). A dropped buffer is freed through the caching
    allocator in stream order, as any tensor."""
    val = cache.get(key)
    if val is None:
        val = cache[key] = make()
        while len(cache) > _CACHED_SHAPES:
            cache.popitem(last=False)
    else:
        cache.move_to_end(key)
    return val


def _block_bytes(b: int, k: int) -> int:
    """One rank's gathered block: b*k int64 ids, then b*k float32 scores, 8-aligned."""
    return (12 * b * k + 7) // 8 * 8


def _block_views(block: torch.Tensor, b: int, k: int):
    """(scores, ids) views of [..., block_bytes] uint8 block(s) as [..., b, k]."""
    n = b * k
    lead = tuple(block.shape[:-1])
    ids = block[..., : 8 * n].view(torch.int64).view(lead + (b, k))
    scores = block[..., 8 * n : 12 * n].view(torch.float32).view(lead + (b, k))
    return scores, ids


def cuda_shard_ops(index: Index) -> ShardOps:
    """Operations backed by this package's kernels for one rank's Index.

    The search workspace is allocated once per (batch, k) and reused by later
    searches of that shape, in stream order on the current stream (the last
    few shapes are kept).
    """
    mod = _ext.load()
    workspaces: OrderedDict = OrderedDict()
    cosine = index.metric == "cosine"

    def workspace(b, kk):
        return _cached(workspaces, (b, kk), lambda: torch.empty(
            max(256, mod.search_workspace_size(b, len(index), index._x.shape[1], kk)), dtype=torch.uint8,
            device=index.device))

    def local_topk_into(queries, k, id_offset, v, i):
        q, release = index._device_queries(queries)
        b = q.shape[0]
        kk = min(k, len(index))
        ws = workspace(b, kk)
        if kk == k:
            mod.search_into(q, index._x, kk, cosine, id_offset, v, i, ws)
        else:  # shard smaller than k: its kk results, then empty slots
            vk = torch.empty((b, kk), dtype=torch.float32, device=index.device)
            ik = torch.empty((b, kk), dtype=torch.int64, device=index.device)
            mod.search_into(q, index._x, kk, cosine, id_offset, vk, ik, ws)
            v[:, :kk] = vk
            i[:, :kk] = ik
            v[:, kk:] = float("-inf")
            i[:, kk:] = -1
        release()

    def local_topk(queries, k, id_offset):
        b = 1 if getattr(queries, "ndim", 2) == 1 else len(queries)
        v = torch.empty((b, k), dtype=torch.float32, device=index.device)
        i = torch.empty((b, k), dtype=torch.int64, device=index.device)
        local_topk_into(queries, k, id_offset, v, i)
        return v, i

    def merge(v_all, i_all, k):
        return mod.merge_lists(v_all, i_all, k)

    return ShardOps(local_topk=local_topk, merge=merge, n_local=len(index), device=index.device,
                    local_topk_into=local_topk_into)


def load_shard_rows(path, rank: int, world: int, metric: str | None = None):
    """(rows, first_row, metric) of shard ``rank`` of ``world`` of a file written
    by ``Index.save``: the contiguous row range [n*rank//world, n*(rank+1)//world)
    of the memory-mapped ``.npy`` (nothing is read until the rows are used) and
    the metric from the ``<path>.json`` sidecar unless given."""
    path = Path(path)
    if metric is None:
        side = Path(str(path) + ".json")
        metric = json.loads(side.read_text())["metric"] if side.exists() else "cosine"
    x = np.load(path, mmap_mode="c")  # copy-on-write: writable for torch, never written back
    n = int(x.shape[0])
    lo, hi = n * rank // world, n * (rank + 1) // world
    return x[lo:hi], lo, metric


class ShardedIndex:
    """Exact top-k over a corpus whose rows are split across the ranks of a group.

    Every rank constructs it collectively with its own contiguous block of rows
    (rank r holds the rows after those of ranks 0..r-1). ``search`` is also
    collective: every rank passes the same queries and receives the same
    (scores [b, k] f32, ids [b, k] i64) with global row ids, best first.
    """

    def __init__(self, shard_embeddings=None, metric: str = "cosine", device=None, group=None,
                 copy: bool = True, ops: ShardOps | None = None):
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("ShardedIndex needs an initialised torch.distributed process group")
        if metric not in ("cosine", "ip"):
            raise ValueError("metric must be 'cosine' or 'ip'")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if ops is None:
            if shard_embeddings is None:
                raise ValueError("shard_embeddings is required")
            x = _to_tensor(shard_embeddings)
            n_local = int(x.shape[0]) if x.dim() == 2 else 0
            size_dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            if size_dev.type == "cuda" and size_dev.index is None:
                size_dev = torch.device("cuda", torch.cuda.current_device())
        else:
            n_local, size_dev = ops.n_local, ops.device
        # Shard sizes first, so that a rank with no rows makes EVERY rank raise
        # the same error here instead of leaving the others blocked in a later
        # collective until the process-group timeout.
        sizes = all_gather_stacked(torch.tensor([n_local], dtype=torch.int64, device=size_dev), group)
        sizes = [int(s) for s in sizes.flatten().tolist()]
        if min(sizes) < 1:
            raise ValueError(f"every rank must hold at least one row; shard sizes are {sizes}")
        if sum(sizes) >= 2**31:
            raise ValueError("a sharded corpus must have fewer than 2^31 rows in total")
        if ops is None:
            self.local = Index(x, metric=metric, device=device, copy=copy)
            ops = cuda_shard_ops(self.local)
        else:
            self.local = None
        self.ops = ops
        self.metric = metric
        self.shard_sizes = sizes
        self.row_offset = sum(sizes[: self.rank])
        self.n_total = sum(sizes)
        self._buffers: OrderedDict = OrderedDict()  # (b, k) -> (local block, gathered blocks), reused in stream order
        # Optional profiling hook: four CUDA events recorded on the current stream
        # before the local search, after it, after the all-gather and after the merge.
        self.phase_events = None

    @classmethod
    def load(cls, path, metric: str | None = None, device=None, group=None, ops_factory=None) -> "ShardedIndex":
        """Collective load of a file written by ``Index.save``: rank r of W maps the
        ``.npy`` and ingests only its contiguous row range [n*r//W, n*(r+1)//W), in
        2^18-row chunks, so no rank reads (or holds) more than its own rows.
        ``ops_factory(rows)``, if given, builds the rank's ShardOps from its rows
        (a numpy array) instead of a GPU Index."""
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("ShardedIndex needs an initialised torch.distributed process group")
        rows, _, metric = load_shard_rows(path, dist.get_rank(group), dist.get_world_size(group), metric)
        if ops_factory is not None:
            return cls(metric=metric, group=group, ops=ops_factory(rows))
        return cls(rows, metric=metric, device=device, group=group)

    def __len__(self) -> int:
        return self.n_total

    def _block_pair(self, b: int, k: int, device):
        def make():
            block = torch.empty(_block_bytes(b, k), dtype=torch.uint8, device=device)
            return block, torch.empty((self.world, block.numel()), dtype=torch.uint8, device=device)

        return _cached(self._buffers, (b, k), make)

    def search(self, queries, k: int = 10):
        k = int(k)
        if k < 1:
            raise ValueError("k must be >= 1")
        k = min(k, self.n_total)
        if k > MAX_FUSED_K:
            raise ValueError(f"sharded search supports k <= {MAX_FUSED_K}")
        ev = self.phase_events
        if ev is not None:
            ev[0].record()
        if self.ops.local_topk_into is not None:
            b = queries.shape[0] if getattr(queries, "ndim", 1) == 2 else 1
            block, gathered = self._block_pair(b, k, self.ops.device)
            v, i = _block_views(block, b, k)
            self.ops.local_topk_into(queries, k, self.row_offset, v, i)
        else:
            v, i = self.ops.local_topk(queries, k, self.row_offset)
            b = v.shape[0]
            block, gathered = self._block_pair(b, k, v.device)
            bv, bi = _block_views(block, b, k)
            bv.copy_(v)
            bi.copy_(i)
        if ev is not None:
            ev[1].record()
        all_gather_stacked(block, self.group, out=gathered)  # [W, block bytes], one collective
        if ev is not None:
            ev[2].record()
        v_all, i_all = _block_views(gathered, b, k)
        out = self.ops.merge(v_all, i_all, k)
        if ev is not None:
            ev[3].record()
        return out
