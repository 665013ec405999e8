"""Exact top-k vector search on NVIDIA B200 (sm_100a) with hand-written kernels.

Drop-in for the reference package's public API (cuda_vector_search/__init__.py:3-7):
``Index``, ``exact_topk_fp32``, ``torch_topk``. ``ShardedIndex`` adds row-sharded
search over a torch.distributed process group (one rank per GPU).
"""

from .index import Index
from .reference import exact_topk_fp32, torch_topk
from .sharded import ShardedIndex

__all__ = ["Index", "ShardedIndex", "exact_topk_fp32", "torch_topk"]
__version__ = "0.1.0"
