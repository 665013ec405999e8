"""numpy restatement of the reference's exact search path (test oracle).

Follows, from the sonhoang/cuda-vector-search sources:
  * exact_topk_fp32  -- cuda_vector_search/reference.py:18-34: fp32 scores of the
    stored fp16 vectors, top-k per chunk of 2^18 rows, ids shifted by the chunk
    start, running merge with the best so far;
  * _normalize_      -- cuda_vector_search/index.py:35-41: rows upcast to fp32,
    divided by max(||row||, 1e-12), rounded back to the storage dtype (fp16);
  * _pad_width       -- cuda_vector_search/index.py:27-32: zero-pad the width to a
    multiple of 64.

The one deliberate addition is a total order on ties: torch.topk leaves the order
of equal scores unspecified, the reference kernels rank score descending then
smaller id first (cuda_vector_search/csrc/kernels.cu:277-279), and so does this
oracle (a stable sort on -score keeps smaller ids first).
"""

from __future__ import annotations

import numpy as np

PAD = 64
CHUNK = 1 << 18


def pad_width(x: np.ndarray) -> np.ndarray:
    """index.py:27-32 -- zero-pad columns to a multiple of 64."""
    d = x.shape[1]
    padded = -(-d // PAD) * PAD
    if padded == d:
        return x
    out = np.zeros((x.shape[0], padded), dtype=x.dtype)
    out[:, :d] = x
    return out


def normalize_rows_fp16(x: np.ndarray) -> np.ndarray:
    """index.py:35-41 on fp16 storage: fp16(fp32(row) / max(||fp32(row)||, 1e-12)).

    The input is first rounded to fp16 (the reference stores to fp16 before it
    normalises, index.py:69-77).
    """
    h = np.asarray(x).astype(np.float16)
    out = np.empty_like(h)
    for start in range(0, h.shape[0], CHUNK):
        blk = h[start : start + CHUNK].astype(np.float32)
        nrm = np.sqrt(np.einsum("ij,ij->i", blk, blk, dtype=np.float32)).astype(np.float32)
        nrm = np.maximum(nrm, np.float32(1e-12))
        out[start : start + CHUNK] = (blk / nrm[:, None]).astype(np.float16)
    return out


def topk_rows(s: np.ndarray, k: int, base: int = 0):
    """Top-k of each row of a score block: (scores desc, ids asc on ties)."""
    k = min(k, s.shape[1])
    if k < s.shape[1]:
        part = np.argpartition(-s, k - 1, axis=1)[:, :k]
        # argpartition may cut through a run of ties at the k-th score; widen to
        # every column tied with it so the stable sort below can pick smallest ids.
        kth = np.take_along_axis(s, part, 1).min(axis=1, keepdims=True)
        cand = [np.nonzero(row >= t)[0] for row, t in zip(s, kth[:, 0])]
    else:
        cand = [np.arange(s.shape[1]) for _ in range(s.shape[0])]
    vals = np.empty((s.shape[0], k), dtype=np.float32)
    ids = np.empty((s.shape[0], k), dtype=np.int64)
    for r, c in enumerate(cand):
        sv = s[r, c]
        order = np.lexsort((c, -sv))[:k]  # primary: score desc, secondary: id asc
        vals[r] = sv[order]
        ids[r] = c[order] + base
    return vals, ids


def merge_topk(v_lists, i_lists, k: int):
    """Best k of concatenated (score, id) lists: score desc, then id asc."""
    v = np.concatenate(v_lists, axis=1)
    i = np.concatenate(i_lists, axis=1)
    k = min(k, v.shape[1])
    order = np.lexsort((i, -v), axis=1)[:, :k] if v.ndim == 2 else None
    return np.take_along_axis(v, order, 1), np.take_along_axis(i, order, 1)


def exact_topk(queries: np.ndarray, corpus: np.ndarray, k: int, chunk: int = CHUNK):
    """reference.py:18-34 in numpy: fp32 scores, chunked top-k with running merge."""
    q = np.asarray(queries, dtype=np.float32)
    best_v = best_i = None
    for start in range(0, corpus.shape[0], chunk):
        blk = np.asarray(corpus[start : start + chunk], dtype=np.float32)
        s = q @ blk.T
        v, i = topk_rows(s, k, base=start)
        if best_v is None:
            best_v, best_i = v, i
        else:
            best_v, best_i = merge_topk([best_v, v], [best_i, i], k)
    return best_v, best_i
