"""The C ABI from a plain C program (tests/c_abi_search.c): no Python or torch
in the search path. The program is compiled here with gcc against
include/cvs.h, libcvs_b200.so and the CUDA runtime, ingests an fp32 corpus,
searches raw fp32 queries twice and writes inputs and results to files; the
results are checked against the CPU oracle on the same fp16-rounded (and, for
cosine, normalised) vectors."""

import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_topk_exact
from oracle import exact_topk, normalize_rows_fp16

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
LIBDIR = ROOT / "cuda-vector-search_b200" / "cuda_vector_search"


def _cuda_home() -> Path:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return Path(nvcc).resolve().parent.parent


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    out = tmp_path_factory.mktemp("cabi") / "c_abi_search"
    cuda = _cuda_home()
    cmd = ["gcc", "-O2", "-std=c11", str(ROOT / "tests" / "c_abi_search.c"), "-o", str(out),
           f"-I{ROOT / 'include'}", f"-I{cuda / 'include'}", f"-L{LIBDIR}", "-l:libcvs_b200.so",
           f"-L{cuda / 'lib64'}", "-lcudart", f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{cuda / 'lib64'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return out


@pytest.mark.parametrize("n,d,b,k,cosine", [(20000, 100, 9, 10, 1), (30000, 384, 200, 64, 0), (5000, 64, 1, 7, 1)])
def test_c_program_search_matches_oracle(program, tmp_path, n, d, b, k, cosine):
    res = subprocess.run([str(program), str(tmp_path), str(n), str(d), str(b), str(k), str(cosine)],
                         capture_output=True, text=True, timeout=300, env=dict(os.environ))
    assert res.returncode == 0, res.stdout + res.stderr
    x = np.fromfile(tmp_path / "corpus.f32", dtype=np.float32).reshape(n, d)
    q = np.fromfile(tmp_path / "queries.f32", dtype=np.float32).reshape(b, d)
    v = np.fromfile(tmp_path / "scores.f32", dtype=np.float32).reshape(b, k)
    i = np.fromfile(tmp_path / "ids.i64", dtype=np.int64).reshape(b, k)
    # The stored vectors: fp16 rounding, then the reference's normalisation for
    # cosine (index.py:35-41; the ingest kernel agrees to within one fp16 ulp,
    # so near-ties are compared at 1e-4 as in the golden-vector tests).
    xs = normalize_rows_fp16(x) if cosine else x.astype(np.float16)
    qs = normalize_rows_fp16(q) if cosine else q.astype(np.float16)
    x32, q32 = xs.astype(np.float32), qs.astype(np.float32)
    ref_v, ref_i = exact_topk(q32, x32, k + 1)
    scale = max(1.0, float(np.abs(ref_v).max()))
    assert_topk_exact(v, i, q32, x32, ref_v, ref_i, k, atol=2e-3 * scale if cosine else 1e-3 * scale,
                      rel=1e-4, scale=1.0)
