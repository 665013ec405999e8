"""The reference's CPU search paths, restated for the timed CPU baseline.

Test and benchmark infrastructure, never part of the product. ``bench.py`` times
these on the GPU box's host cores next to the B200 numbers (its ``cpu_baseline``
field and its ``--impl reference`` arm); the reference package itself cannot
travel to that box. Each function follows a file of sonhoang/cuda-vector-search:

  * index_cpu_search      -- ``Index(..., device="cpu").search``: the CPU index
    stores fp32 rows (cuda_vector_search/index.py:66-78) and ``search`` falls to
    ``torch_topk`` (index.py:117-131 -> reference.py:8-15): one fp32
    ``torch.matmul`` for the whole [b, n] score matrix, then ``torch.topk``;
  * torch_exact_topk_fp32 -- ``exact_topk_fp32`` (reference.py:18-34): fp32 scores
    per chunk of 2^18 rows, top-k per chunk, ids shifted by the chunk start,
    running merge with torch.cat / topk / gather;
  * numpy_search          -- ``numpy_search`` of bench/bench_baselines.py:45-50:
    one fp32 matmul, argpartition, then a sort of the k survivors;
  * time_call             -- bench/timing.py:9-34: median wall time after a
    warm-up, repeated until a time budget or a repetition cap is reached.

The functions keep the reference's arithmetic (fp32 scores of the given
vectors), so their outputs agree with ``oracle.exact_topk`` up to the order of
exactly equal scores; tests/test_oracle.py checks that.
"""

from __future__ import annotations

import statistics
import time

import numpy as np
import torch


def index_cpu_search(queries: torch.Tensor, corpus: torch.Tensor, k: int):
    """reference index.py:131 / reference.py:8-15 on fp32 CPU tensors."""
    s = queries @ corpus.T
    v, i = torch.topk(s, k, dim=1)
    return v.float(), i


def torch_exact_topk_fp32(queries: torch.Tensor, corpus: torch.Tensor, k: int, chunk: int = 1 << 18):
    """reference.py:18-34: chunked fp32 top-k with a running merge."""
    q = queries.float()
    best_v = best_i = None
    for start in range(0, corpus.shape[0], chunk):
        s = q @ corpus[start : start + chunk].float().T
        v, i = torch.topk(s, min(k, s.shape[1]), dim=1)
        i = i + start
        if best_v is None:
            best_v, best_i = v, i
            continue
        v = torch.cat([best_v, v], dim=1)
        i = torch.cat([best_i, i], dim=1)
        best_v, sel = torch.topk(v, min(k, v.shape[1]), dim=1)
        best_i = torch.gather(i, 1, sel)
    return best_v, best_i


def numpy_search(q: np.ndarray, x: np.ndarray, k: int):
    """bench/bench_baselines.py:45-50: matmul, argpartition, sort the survivors."""
    s = q @ x.T
    part = np.argpartition(-s, k - 1, axis=1)[:, :k]
    pv = np.take_along_axis(s, part, 1)
    order = np.argsort(-pv, axis=1)
    return np.take_along_axis(pv, order, 1), np.take_along_axis(part, order, 1)


def time_call(fn, target_s: float = 0.3, max_reps: int = 100, warmup: int = 2, slow_s: float = 1.0):
    """bench/timing.py:9-34: (median milliseconds, repetitions) of fn().

    ``warmup`` calls first (only the first one if it took longer than ``slow_s``),
    then repetitions until ``target_s`` seconds have run (at least three) or
    ``max_reps``; a repetition longer than ``slow_s`` ends the loop.
    """

    def once():
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    first = once()
    if first < slow_s:
        for _ in range(warmup - 1):
            once()
    times = []
    total = 0.0
    while len(times) < max_reps and (total < target_s or len(times) < 3):
        dt = once()
        times.append(dt)
        total += dt
        if dt > slow_s:
            break
    return 1000.0 * statistics.median(times), len(times)
