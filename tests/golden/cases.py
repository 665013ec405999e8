"""Seeded test cases shared by the golden-vector generator and the tests.

``make`` restates the reference's test input generator (tests/test_search.py:11-18
of sonhoang/cuda-vector-search): one CPU torch.Generator seeded per case, corpus
then queries drawn from it with randn, optional row L2 normalisation, rounded to
fp16. ``scale_rows`` varies the row norms the way the reference's cosine test does
(tests/test_search.py:86), but draws from the same seeded generator so the
inputs are reproducible.
"""

from __future__ import annotations

import torch


def make(n, d, b, seed=0, normal=True, scale_rows=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    q = torch.randn(b, d, generator=g)
    if normal:
        x = x / x.norm(dim=1, keepdim=True)
        q = q / q.norm(dim=1, keepdim=True)
    x, q = x.half(), q.half()
    if scale_rows:
        x = x * torch.rand(n, 1, generator=g).half() * 4
    return x, q


def _case(name, n, d, b, k, seed, metric="ip", normal=True, **kw):
    c = dict(name=name, n=n, d=d, b=b, k=k, seed=seed, metric=metric, normal=normal)
    c.update(kw)
    return c


# tests/test_search.py:50-62 (ip on unit vectors, seed = n + d + b + k)
FUSED = [
    (1000, 64, 1, 1),
    (1000, 64, 3, 10),
    (4099, 128, 17, 10),
    (20000, 384, 1, 10),
    (20000, 384, 32, 100),
    (20000, 384, 100, 33),
    (20000, 768, 256, 64),
    (50000, 384, 70, 128),
    (30000, 384, 40, 256),
    (300, 96, 5, 150),
    (100, 64, 2, 100),
]

CASES = [_case(f"fused_{n}_{d}_{b}_{k}", n, d, b, k, n + d + b + k) for n, d, b, k in FUSED]
# tests/test_search.py:73 (twopass / torch paths, seed 3)
CASES += [_case(f"twopass_{n}_{d}_{b}_{k}", n, d, b, k, 3) for n, d, b, k in [(5000, 384, 8, 10), (20000, 768, 64, 100)]]
# tests/test_search.py:84-92 (cosine, unnormalised input with varied norms)
CASES += [_case("cosine_unnormalised", 8000, 384, 16, 10, 7, metric="cosine", normal=False, scale_rows=True)]
# tests/test_search.py:96-100 (raw inner product, |s| ~ 16-60)
CASES += [_case("raw_ip_large", 10000, 256, 9, 50, 11, normal=False)]
# tests/test_search.py:104-113 (score matrix)
CASES += [_case("scores_3001_192_37", 3001, 192, 37, 10, 5)]
# tests/test_search.py:117-121 (chunked fp32 helper)
CASES += [_case("exact_helper", 70000, 128, 4, 20, 9, chunk=8192)]
# tests/test_search.py:135-143 (plan overrides)
CASES += [_case("plan_overrides", 40000, 384, 50, 10, 4)]
# tests/test_search.py:160-168 (large per-list state)
CASES += [_case(f"large_state_{k}_{bq}", 30000, 384, 70, k, k + bq, bq=bq) for k, bq in [(100, 64), (256, 32), (200, 16), (40, 64)]]
# Added here: GEMV batches (b <= 8), odd widths, cosine with padding, ragged tiles.
CASES += [
    _case("gemv_1_768_10", 20000, 768, 1, 10, 101),
    _case("gemv_2_768_32", 20000, 768, 2, 32, 102),
    _case("gemv_3_384_17", 20011, 384, 3, 17, 103),
    _case("gemv_5_1024_10", 9000, 1024, 5, 10, 104),
    _case("gemv_8_768_32", 20000, 768, 8, 32, 105),
    _case("cosine_pad_100", 4096, 100, 12, 7, 21, metric="cosine", normal=False),
    _case("ragged_129_1000", 12345, 1000, 129, 16, 22),
    _case("wide_1536", 3000, 1536, 20, 10, 23),
]

BY_NAME = {c["name"]: c for c in CASES}
