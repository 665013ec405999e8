"""Parity checks shared by the tests (test infrastructure).

`assert_topk_exact` combines the reference's exactness contract
(tests/test_search.py:21-44 of sonhoang/cuda-vector-search: ids in range and
unique, rows sorted, every returned id scores at least the true k-th minus a
tolerance, returned scores equal their ids' fp32 scores) with the stricter rule
this build is held to: returned ids equal the fp32 oracle's top-k except where the
oracle's k-th and (k+1)-th scores differ by less than 1e-5 relative, and scores
agree within 1e-3 absolute.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
REL_TIE = 1e-5
ATOL = 1e-3


def golden(name: str):
    meta = json.loads((GOLDEN / "golden.json").read_text())[name]
    z = np.load(GOLDEN / f"{name}.npz")
    return meta, z["scores"], z["ids"]


def true_scores(q32: np.ndarray, x32: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """fp32 score of each returned id: q[r] . x[ids[r, j]]."""
    out = np.empty(ids.shape, dtype=np.float64)
    for r in range(ids.shape[0]):
        out[r] = x32[ids[r]].astype(np.float64) @ q32[r].astype(np.float64)
    return out


def assert_topk_exact(got_v, got_i, q32, x32, ref_v, ref_i, k, atol=ATOL, rel=REL_TIE, scale=None):
    """got_*: [b, k] results. ref_*: oracle top-(k+1) (top-k when k == n)."""
    got_v = np.asarray(got_v, dtype=np.float64)
    got_i = np.asarray(got_i, dtype=np.int64)
    n = x32.shape[0]
    b = q32.shape[0]
    assert got_v.shape == (b, k) and got_i.shape == (b, k), (got_v.shape, got_i.shape, (b, k))
    assert (got_i >= 0).all() and (got_i < n).all(), "ids out of range"
    ts = true_scores(q32, x32, got_i)
    if scale is None:
        scale = 1.0
    err = np.abs(got_v - ts).max()
    assert err <= atol * scale, f"scores do not match their ids (max err {err})"
    for r in range(b):
        row = got_i[r]
        assert len(set(row.tolist())) == k, f"duplicate ids in row {r}"
        gv = got_v[r]
        assert (gv[:-1] >= gv[1:]).all(), f"row {r} not sorted"
        eq = gv[:-1] == gv[1:]
        assert (row[:-1][eq] < row[1:][eq]).all(), f"row {r}: equal scores not ordered by id"
        kth = float(ref_v[r, k - 1])
        tol = rel * max(abs(kth), 1e-30)
        assert (ts[r] >= kth - max(tol, 1e-6 * scale)).all(), f"row {r}: an id outside the true top-{k}"
        boundary_tie = ref_v.shape[1] > k and abs(float(ref_v[r, k - 1]) - float(ref_v[r, k])) < tol
        if not boundary_tie:
            missing = set(ref_i[r, :k].tolist()) - set(row.tolist())
            assert not missing, f"row {r}: ids {sorted(missing)[:5]} of the oracle top-{k} missing"


class DeviceRows:
    """The stored corpus of an index, read row by row for ``assert_topk_exact``.

    Stands in for the host fp32 matrix at sizes that do not fit in host memory
    at once: ``shape`` is [n, d] and ``rows[ids]`` copies the requested stored
    fp16 rows from the device and widens them to fp32 (exact).
    """

    def __init__(self, x_dev, d: int):
        self.x = x_dev
        self.d = d
        self.shape = (int(x_dev.shape[0]), d)

    def __getitem__(self, ids):
        import torch

        t = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=self.x.device)
        return self.x.index_select(0, t).cpu()[:, : self.d].float().numpy()


def device_blocks(x_dev, d: int, rows: int = 1 << 19):
    """(first_row, fp32 host rows) blocks of a stored device corpus, for
    ``oracle.exact_topk_blocks``: fp16 rows copied to the host, widened to fp32."""
    for start in range(0, int(x_dev.shape[0]), rows):
        blk = x_dev[start : start + rows].cpu()
        yield start, blk[:, :d].float().numpy()
