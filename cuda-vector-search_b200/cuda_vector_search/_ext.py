"""Access to the prebuilt native extension (no JIT build, no fallback).

Mirrors the reference loader's interface (cuda_vector_search/_ext.py:15-47):
``available()`` and a thread-safe ``load()`` returning the extension module with
``scores`` and ``fused_topk``. The module is built in-tree by
``cuda-vector-search_b200/build.py`` for sm_100a only; on anything else
``load()`` raises RuntimeError instead of falling back.
"""

from __future__ import annotations

import threading

_lock = threading.Lock()
_mod = None


def available() -> bool:
    """True when a CUDA device with compute capability 10.0 (B200) is present."""
    import torch

    if not torch.cuda.is_available():
        return False
    return tuple(torch.cuda.get_device_capability()) == (10, 0)


def load(verbose: bool = False):
    """Return the extension module (imported once, under a lock)."""
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        if not available():
            raise RuntimeError("cuda-vector-search B200 kernels need an sm_100 (B200) CUDA GPU")
        try:
            from . import _C  # noqa: PLC0415
        except ImportError as e:  # pragma: no cover - depends on the build
            raise RuntimeError(
                "the native extension is not built; run `python cuda-vector-search_b200/build.py`"
            ) from e
        if verbose:
            print("cuda_vector_search: loaded", _C.__file__)
        _mod = _C
        return _mod
