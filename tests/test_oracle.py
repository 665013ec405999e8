"""The CPU oracle pinned against the reference's own outputs (golden vectors)."""

import hashlib

import numpy as np
import pytest
import torch

from cases import CASES, make
from helpers import assert_topk_exact, golden
from oracle import exact_topk, normalize_rows_fp16

SMALL = [c for c in CASES if c["n"] * c["d"] <= 30000 * 1536]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", SMALL, ids=lambda c: c["name"])
def test_inputs_reproduce(case):
    """The seeded generator yields the inputs the golden vectors were made from."""
    meta, _, _ = golden(case["name"])
    x, q = make(case["n"], case["d"], case["b"], seed=case["seed"], normal=case["normal"],
                scale_rows=case.get("scale_rows", False))
    assert sha(x.numpy()) == meta["x_sha"]
    assert sha(q.numpy()) == meta["q_sha"]


@pytest.mark.parametrize("case", SMALL, ids=lambda c: c["name"])
def test_oracle_matches_reference(case):
    meta, ref_v, ref_i = golden(case["name"])
    x, q = make(case["n"], case["d"], case["b"], seed=case["seed"], normal=case["normal"],
                scale_rows=case.get("scale_rows", False))
    x, q = x.numpy(), q.numpy()
    rel = 1e-5
    if case["metric"] == "cosine":
        # torch's CPU norm is not correctly rounded, so a few elements of the
        # reference's normalised rows differ by one fp16 ulp from this
        # restatement (test_normalize_matches_torch_reference_formula bounds it);
        # scores then move by ~1e-5, so near-ties are compared at 1e-4 here.
        x, q = normalize_rows_fp16(x), normalize_rows_fp16(q)
        rel = 1e-4
    k = min(case["k"], case["n"])
    v, i = exact_topk(q, x, min(k + 1, case["n"]), chunk=case.get("chunk", 1 << 18))
    assert np.abs(v[:, :k] - ref_v[:, :k]).max() < rel * max(1.0, np.abs(ref_v).max())
    assert_topk_exact(v[:, :k], i[:, :k], q.astype(np.float32), x.astype(np.float32), ref_v, ref_i, k,
                      rel=rel)


def test_chunked_merge_equals_one_shot():
    """reference tests/test_search.py:116-121 on the oracle."""
    x, q = make(70000, 128, 4, seed=9)
    v1, i1 = exact_topk(q.numpy(), x.numpy(), 20, chunk=8192)
    v2, i2 = exact_topk(q.numpy(), x.numpy(), 20, chunk=1 << 20)
    assert np.abs(v1 - v2).max() < 1e-5
    assert (i1 == i2).all()


def test_oracle_tie_order():
    """Duplicated rows: equal scores come back smallest id first."""
    rng = np.random.default_rng(5)
    base = rng.standard_normal((7, 64)).astype(np.float16)
    x = np.repeat(base, 4, axis=0)
    q = rng.standard_normal((3, 64)).astype(np.float16)
    v, i = exact_topk(q, x, 9, chunk=5)
    for r in range(3):
        for j in range(8):
            if v[r, j] == v[r, j + 1]:
                assert i[r, j] < i[r, j + 1]


@pytest.mark.parametrize("case", [c for c in CASES if c["metric"] == "cosine"], ids=lambda c: c["name"])
def test_normalize_matches_reference(case):
    """index.py:35-41 of the reference, run here through torch on the same fp16 rows."""
    x, q = make(case["n"], case["d"], case["b"], seed=case["seed"], normal=case["normal"],
                scale_rows=case.get("scale_rows", False))
    ours = normalize_rows_fp16(x.numpy())
    blk = x.float()
    ref = (blk / blk.norm(dim=1, keepdim=True).clamp_min(1e-12)).half()
    meta, _, _ = golden(case["name"])
    assert sha(ref.numpy()) == meta["xn_sha"]  # this formula is the reference's _normalize_
    diff = np.abs(ours.view(np.int16).astype(np.int32) - ref.numpy().view(np.int16).astype(np.int32))
    assert diff.max() <= 1  # at most one fp16 ulp
    assert (diff == 0).mean() > 0.9999


def test_cpu_baseline_paths_agree_with_the_oracle():
    """The three timed CPU paths (oracle/cpu_paths.py) compute the reference's
    fp32 search: same top-k as the oracle on the same stored vectors."""
    from oracle import compare_topk, index_cpu_search, numpy_search, time_call, torch_exact_topk_fp32

    x, q = make(30000, 128, 6, seed=3)
    x32, q32 = x.float(), q.float()
    ref_v, ref_i = exact_topk(q.numpy(), x.numpy(), 11)
    for v, i in (index_cpu_search(q32, x32, 10), torch_exact_topk_fp32(q32, x32, 10, chunk=7000),
                 numpy_search(q32.numpy(), x32.numpy(), 10)):
        res = compare_topk(np.asarray(v), np.asarray(i), ref_v, ref_i, 10, atol=1e-5)
        assert res["ok"] and res["recall"] == 1.0, res
    ms, reps = time_call(lambda: numpy_search(q32.numpy(), x32.numpy(), 10), target_s=0.05)
    assert ms > 0 and reps >= 3


def test_streamed_blocks_equal_one_shot():
    """exact_topk_blocks over uneven blocks in any order equals exact_topk."""
    from oracle import exact_topk_blocks

    x, q = make(20000, 64, 5, seed=8)
    xs = x.numpy()
    bounds = [0, 777, 5000, 5001, 13000, 20000]
    blocks = [(bounds[j], xs[bounds[j]:bounds[j + 1]]) for j in range(len(bounds) - 1)][::-1]
    v1, i1 = exact_topk_blocks(q.numpy(), iter(blocks), 15)
    v2, i2 = exact_topk(q.numpy(), xs, 15)
    assert (i1 == i2).all() and np.abs(v1 - v2).max() < 1e-6


def test_compare_topk_flags_a_wrong_id():
    from oracle import compare_topk

    x, q = make(5000, 64, 4, seed=2)
    ref_v, ref_i = exact_topk(q.numpy(), x.numpy(), 11)
    got_v, got_i = ref_v[:, :10].copy(), ref_i[:, :10].copy()
    assert compare_topk(got_v, got_i, ref_v, ref_i, 10)["ok"]
    got_i[2, 9] = ref_i[2, 10] + 1 if ref_i[2, 10] + 1 not in ref_i[2] else 4999
    assert compare_topk(got_v, got_i, ref_v, ref_i, 10)["bad_rows"] == [2]
    got_i[2, 9] = ref_i[2, 9]
    got_v[1, 0] += 0.01
    assert not compare_topk(got_v, got_i, ref_v, ref_i, 10)["ok"]
