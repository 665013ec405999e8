"""CPU oracle for parity tests -- test infrastructure, never part of the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline. The product path (``cuda_vector_search``)
never imports it and has no CPU fallback.

Pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference package and records its
``exact_topk_fp32`` and ``_normalize_`` outputs); ``tests/test_oracle.py`` checks
this restatement against those fixtures.
"""

from .exact import exact_topk, merge_topk, normalize_rows_fp16, pad_width, topk_rows

__all__ = ["exact_topk", "merge_topk", "normalize_rows_fp16", "pad_width", "topk_rows"]
