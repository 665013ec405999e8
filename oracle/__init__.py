"""CPU oracle for parity tests -- test infrastructure, never part of the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` may import this
package: tests and smoke() as the checker; bench.py for its ``cpu_baseline`` /
``--impl reference`` legs (the timed CPU baseline, ``cpu_paths``) and for the
``parity`` check it runs after its timed loops (a checker, outside every timed
region). The product path (``cuda_vector_search``) never imports it and has no
CPU fallback.

Pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference package and records its
``exact_topk_fp32`` and ``_normalize_`` outputs); ``tests/test_oracle.py`` checks
this restatement against those fixtures.
"""

from .cpu_paths import index_cpu_search, numpy_search, time_call, torch_exact_topk_fp32
from .exact import (compare_topk, exact_topk, exact_topk_blocks, merge_topk, normalize_rows_fp16, pad_width,
                    topk_rows)

__all__ = ["compare_topk", "exact_topk", "exact_topk_blocks", "index_cpu_search", "merge_topk",
           "normalize_rows_fp16", "numpy_search", "pad_width", "time_call", "topk_rows", "torch_exact_topk_fp32"]
