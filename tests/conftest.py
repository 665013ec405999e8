"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs here without a GPU (oracle vs golden vectors, C-ABI exports,
host logic, gloo multi-rank logic). `-m gpu` runs the parity tests on a B200.
"""

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "cuda-vector-search_b200", ROOT / "tests" / "golden", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 4))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
