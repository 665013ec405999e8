"""Exact top-k search over an fp16 embedding matrix held on one B200.

Same public API as the reference's ``cuda_vector_search.Index``
(cuda_vector_search/index.py:44-155): constructor arguments, ``search``,
``scores``, ``save`` / ``load``, ``len()``, ``.dim``, ``.embeddings``. What changes
underneath:

* storage: one ingest kernel converts to fp16, L2-normalises (cosine) and pads
  the width to a multiple of 64 in a single pass (index.py:35-41 + 27-32 there);
* search: ``method="fused"`` (the default) is three launches: the queries'
  preparation (to fp16, normalised for cosine, padded) fused with the
  workspace clear, the tcgen05 score + top-k kernel (or the GEMV kernel for a
  single query, and for up to 8 queries on a small corpus), and a merge kernel; queries in pinned host memory are copied
  on a side stream, so a caller that issues the next search before reading
  back the previous results overlaps each upload with the previous search (a
  fixed ring of device buffers, nothing allocated per call);
* there is no CPU storage and no fallback: a non-CUDA device or a GPU other than
  sm_100 raises RuntimeError. ``method="torch"`` (cuBLAS + topk) remains available
  on request, as in the reference.
"""

from __future__ import annotations

import json
import threading
from pathlib import Path

import numpy as np
import torch

from . import _ext
from .reference import torch_topk

PAD = 64  # width granularity (reference index.py:14)
MAX_FUSED_K = 1024  # reference: 256 (index.py:15); larger k runs on the same kernels here
_INGEST_CHUNK = 1 << 18  # rows staged per host->device copy

METHODS = ("auto", "fused", "twopass", "torch")

_KERNEL_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)

_SIDE_UPLOAD_BYTES = 256 << 10  # smaller pinned uploads stay on the current stream
_RING_MAX_BYTES = 32 << 20  # larger pinned blocks (bulk corpus ingest) use the allocator
_RING_SLOTS = 4


class _UploadRing:
    """Fixed device buffers for pinned host uploads, refilled round-robin.

    Each upload is copied on a side stream into the next slot; the current stream
    waits for the copy (an event, no host synchronisation), so the copy runs while
    the current stream's earlier kernels (the previous search) still execute. A
    slot is refilled only after the ingest kernel that read its previous contents
    has run (the side stream waits on an event recorded after that kernel). No
    memory is allocated per call: growing the caching allocator's pool for a side
    stream took cudaMalloc calls that stalled the host for milliseconds.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.side = torch.cuda.Stream(device=device)
        self.bufs: list = [None] * _RING_SLOTS
        self.consumed = [torch.cuda.Event() for _ in range(_RING_SLOTS)]
        self.used = [False] * _RING_SLOTS
        self.next = 0
        self.lock = threading.Lock()

    def upload(self, blk: torch.Tensor):
        """Copy pinned ``blk`` into the next slot on the side stream; the current
        stream waits for the copy. Returns the device copy and a callable to run
        once the kernels that read it are enqueued (it marks the slot reusable
        after them)."""
        cur = torch.cuda.current_stream(self.device)
        nelem = blk.numel()
        with self.lock:
            j = self.next
            self.next = (j + 1) % _RING_SLOTS
            if self.used[j]:
                self.side.wait_event(self.consumed[j])
            buf = self.bufs[j]
            if buf is None or buf.dtype != blk.dtype or buf.numel() < nelem:
                if buf is not None:
                    # Queued work on the current stream may still read it.
                    buf.record_stream(cur)
                with torch.cuda.stream(self.side):
                    buf = self.bufs[j] = torch.empty(nelem, dtype=blk.dtype, device=self.device)
            dst = buf[:nelem].view(blk.shape)
            with torch.cuda.stream(self.side):
                dst.copy_(blk, non_blocking=True)
            cur.wait_stream(self.side)
            self.used[j] = True

        def release():
            self.consumed[j].record(cur)

        return dst, release

    def ingest(self, blk: torch.Tensor, out: torch.Tensor, cosine: bool, mod) -> None:
        """Upload pinned ``blk`` and run the ingest kernel from it into ``out``."""
        dst, release = self.upload(blk)
        mod.ingest_into(dst, out, cosine)
        release()


_RINGS: dict = {}  # device index -> _UploadRing
_RINGS_LOCK = threading.Lock()


def _nothing() -> None:
    pass


def _upload_ring(device: torch.device) -> _UploadRing:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ring = _RINGS.get(idx)
    if ring is None:
        with _RINGS_LOCK:
            ring = _RINGS.get(idx)
            if ring is None:
                ring = _RINGS[idx] = _UploadRing(torch.device("cuda", idx))
    return ring


def _to_tensor(a) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a
    return torch.from_numpy(np.ascontiguousarray(a))


def pad_width(d: int) -> int:
    return -(-int(d) // PAD) * PAD


def _ingest(src: torch.Tensor, device: torch.device, cosine: bool, out: torch.Tensor | None = None):
    """fp16, optionally L2-normalised, width-padded copy of ``src`` on ``device``.

    ``src`` may live on the host (staged through in chunks) or on the device. When
    ``out`` is ``src`` itself the rows are normalised in place.
    """
    mod = _ext.load()
    if src.dtype not in _KERNEL_DTYPES:
        src = src.to(torch.float32)
    n, d = src.shape
    if out is None:
        out = torch.empty((n, pad_width(d)), dtype=torch.float16, device=device)
    if n == 0:
        return out
    if src.device == device:
        if src.stride(1) != 1:
            src = src.contiguous()
        mod.ingest_into(src, out, cosine)
        return out
    # Host source: stage fixed-size row blocks so a huge array never needs a
    # second full-size copy on either side. Contiguous pinned blocks of at least
    # _SIDE_UPLOAD_BYTES go through the upload ring's side stream (the extra host
    # work of the stream switch outweighs the overlap for small ones).
    pinned = src.is_pinned()
    with torch.cuda.device(device):
        for start in range(0, n, _INGEST_CHUNK):
            blk = src if n <= _INGEST_CHUNK else src[start : start + _INGEST_CHUNK]
            dst = out if n <= _INGEST_CHUNK else out[start : start + blk.shape[0]]
            if pinned and _SIDE_UPLOAD_BYTES <= blk.nbytes <= _RING_MAX_BYTES and blk.is_contiguous():
                _upload_ring(device).ingest(blk, dst, cosine, mod)
                continue
            blk_dev = blk.to(device, non_blocking=pinned)
            if blk_dev.stride(1) != 1:
                blk_dev = blk_dev.contiguous()
            mod.ingest_into(blk_dev, dst, cosine)
    return out


class Index:
    """Brute-force (exact) top-k index on one B200.

    Args:
        embeddings: [n, d] array or tensor (any float dtype; host or device).
            Stored as fp16 rows zero-padded to a multiple of 64 columns.
        metric: "cosine" (rows and queries are L2-normalised) or "ip" (raw inner product).
        device: "cuda", "cuda:1", ...; defaults to the current CUDA device. Only
            CUDA devices of compute capability 10.0 are supported.
        copy: if False and ``embeddings`` is already a contiguous fp16 tensor on
            ``device`` whose width is a multiple of 64, it is used as-is (and
            normalised in place for cosine).
    """

    def __init__(self, embeddings, metric: str = "cosine", device=None, copy: bool = True):
        if metric not in ("cosine", "ip"):
            raise ValueError("metric must be 'cosine' or 'ip'")
        x = _to_tensor(embeddings)
        if x.dim() != 2:
            raise ValueError("embeddings must be 2-D [n, d]")
        if x.shape[0] == 0:
            raise ValueError("embeddings is empty")
        if device is None:
            if not torch.cuda.is_available():
                raise RuntimeError("cuda_vector_search (B200 build) needs a CUDA device; none is available")
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("cuda_vector_search (B200 build) stores the index on a CUDA device only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        _ext.load()  # raises unless the sm_100 extension is usable
        self.metric = metric
        self.dim = int(x.shape[1])
        if x.shape[0] >= 2**31 - 1:
            raise ValueError("embeddings must have fewer than 2^31 - 1 rows")
        cosine = metric == "cosine"
        in_place = (
            not copy
            and x.device == self.device
            and x.dtype == torch.float16
            and x.is_contiguous()
            and self.dim % PAD == 0
        )
        self._x = _ingest(x, self.device, cosine, out=x if in_place else None)
        self._use_kernels = True

    # -- basics -------------------------------------------------------------
    def __len__(self) -> int:
        return int(self._x.shape[0])

    @property
    def embeddings(self) -> torch.Tensor:
        """The stored matrix (normalised for cosine), without padding."""
        return self._x[:, : self.dim]

    def _device_queries(self, queries):
        """Raw queries as a 2-D tensor on the index device with contiguous rows,
        not yet converted, normalised or padded (the search's first launch does
        that), and a callable to run once the search is enqueued. Pinned host
        queries of 256 KB and more are copied on the upload ring's side stream."""
        q = self._query_tensor(queries)
        if q.dtype not in _KERNEL_DTYPES:
            q = q.to(torch.float32)
        if q.device == self.device:
            return (q if q.stride(1) == 1 else q.contiguous()), _nothing
        if q.is_pinned() and q.is_contiguous() and _SIDE_UPLOAD_BYTES <= q.nbytes <= _RING_MAX_BYTES:
            with torch.cuda.device(self.device):
                return _upload_ring(self.device).upload(q)
        q = q.to(self.device, non_blocking=q.is_pinned())
        return (q if q.stride(1) == 1 else q.contiguous()), _nothing

    def _query_tensor(self, queries) -> torch.Tensor:
        """The queries as a 2-D tensor, validated like the reference (index.py:89-94)."""
        q = _to_tensor(queries)
        if q.dim() == 1:
            q = q[None]
        if q.dim() != 2 or q.shape[1] != self.dim:
            raise ValueError(f"queries must be [b, {self.dim}]")
        return q

    def _prep_queries(self, queries) -> torch.Tensor:
        return _ingest(self._query_tensor(queries), self.device, self.metric == "cosine")

    # -- search -------------------------------------------------------------
    def search(self, queries, k: int = 10, method: str = "auto"):
        """Return (scores [b, k] float32, ids [b, k] int64), best first.

        method:
            "fused"   - tcgen05 (or GEMV for b = 1, and b <= 8 on small corpora) scores + top-k
                        in one pass (k <= 1024)
            "twopass" - score kernel writes the full matrix, then torch.topk
            "torch"   - torch.matmul (cuBLAS) + torch.topk
            "auto"    - fused when k <= 1024, else twopass
        """
        if method not in METHODS:
            raise ValueError(f"method must be one of {METHODS}")
        k = int(k)
        if k < 1:
            raise ValueError("k must be >= 1")
        k = min(k, len(self))
        if method == "auto":
            method = "fused" if k <= MAX_FUSED_K else "twopass"
        mod = _ext.load()
        if method == "fused":
            if k > MAX_FUSED_K:
                self._query_tensor(queries)  # the reference reports bad queries first
                raise ValueError(f"fused search supports k <= {MAX_FUSED_K}")
            q, release = self._device_queries(queries)
            # Query preparation, workspace clear, search and merge: three launches.
            v, i = mod.search(q, self._x, k, self.metric == "cosine")
            release()
            return v, i
        q = self._prep_queries(queries)
        if method == "twopass":
            s = mod.scores(q, self._x, False)
            v, i = torch.topk(s, k, dim=1)
            return v.float(), i
        return torch_topk(q, self._x, k)

    def scores(self, queries, fp32: bool = True) -> torch.Tensor:
        """Full [b, n] score matrix from the tcgen05 score kernel."""
        q = self._prep_queries(queries)
        return _ext.load().scores(q, self._x, fp32)

    # -- persistence --------------------------------------------------------
    def save(self, path) -> None:
        """Write the stored vectors to `path` (.npy, fp16) plus a small `<path>.json` sidecar."""
        path = Path(path)
        np.save(path, self.embeddings.to(torch.float16).cpu().numpy())
        meta = {"metric": self.metric, "dim": self.dim, "n": len(self)}
        Path(str(path) + ".json").write_text(json.dumps(meta))

    @classmethod
    def load(cls, path, metric: str | None = None, device=None) -> "Index":
        """Read a file written by ``save`` (reference index.py:148-155).

        The ``.npy`` is memory-mapped, not read whole: the ingest stages it to the
        device in 2^18-row chunks, so host memory holds one chunk at a time.
        """
        path = Path(path)
        if metric is None:
            side = Path(str(path) + ".json")
            metric = json.loads(side.read_text())["metric"] if side.exists() else "cosine"
        # Copy-on-write mapping: writable for torch.from_numpy, never written back.
        x = np.load(path, mmap_mode="c")
        return cls(x, metric=metric, device=device, copy=False)
