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
    blocks = ((start, corpus[start : start + chunk]) for start in range(0, corpus.shape[0], chunk))
    return exact_topk_blocks(queries, blocks, k)


def exact_topk_blocks(queries: np.ndarray, blocks, k: int):
    """The same chunked search over corpus blocks supplied by the caller.

    ``blocks`` yields ``(first_row, rows)`` pairs that together cover the corpus
    (any block size, in any order); ``rows`` is converted to fp32. This lets a
    checker stream a corpus that does not fit in host memory at once (e.g. from
    device memory) through the same arithmetic as ``exact_topk``: per block fp32
    scores and top-k with ids shifted by the block start, then the running merge
    of reference.py:28-33. The result does not depend on the block size: ties are
    ordered by id.
    """
    q = np.asarray(queries, dtype=np.float32)
    best_v = best_i = None
    for start, rows in blocks:
        blk = np.asarray(rows, dtype=np.float32)
        s = q @ blk.T
        v, i = topk_rows(s, k, base=start)
        if best_v is None:
            best_v, best_i = v, i
        else:
            best_v, best_i = merge_topk([best_v, v], [best_i, i], k)
    return best_v, best_i


def compare_topk(got_v, got_i, ref_v, ref_i, k: int, atol: float = 1e-3, rel: float = 1e-5) -> dict:
    """Checks a [b, k] search result against the oracle's top-(k+1) (top-k when k == n).

    The acceptance rule of the fused path: every returned id is one of the
    oracle's top-k ids, except where the oracle's k-th and (k+1)-th scores are
    closer than ``rel`` (relative), and every returned score is within ``atol``
    of the oracle's score at the same rank. Rows must come back best first.
    Returns {"ok", "rows", "recall", "max_abs_err", "bad_rows"}.
    """
    got_v = np.asarray(got_v, dtype=np.float64)
    got_i = np.asarray(got_i, dtype=np.int64)
    ref_v = np.asarray(ref_v, dtype=np.float64)
    ref_i = np.asarray(ref_i, dtype=np.int64)
    b = got_v.shape[0]
    hits = 0
    bad = []
    err = float(np.abs(got_v - ref_v[:, :k]).max()) if b else 0.0
    for r in range(b):
        want = set(ref_i[r, :k].tolist())
        hit = len(want & set(got_i[r].tolist()))
        hits += hit
        tie = ref_v.shape[1] > k and abs(ref_v[r, k - 1] - ref_v[r, k]) < rel * max(abs(ref_v[r, k - 1]), 1e-30)
        if (hit < k and not tie) or not (got_v[r, :-1] >= got_v[r, 1:]).all():
            bad.append(r)
    return {"ok": not bad and err <= atol, "rows": int(b), "recall": hits / max(1, b * k),
            "max_abs_err": err, "bad_rows": bad[:8]}
