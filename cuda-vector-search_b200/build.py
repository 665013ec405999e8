"""Build the native parts in-tree.

    python cuda-vector-search_b200/build.py [--force] [--verbose]

Produces, inside the package directory cuda_vector_search/:
  libcvs_b200.so          the C-ABI library (include/cvs.h), sm_100a kernels,
                          CUDA runtime linked statically, no torch dependency;
  _C<ext suffix>          the thin PyTorch binding over that library.

Object files go to _build/ (git-ignored). A target is rebuilt only when one of
its sources or headers is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
PKG = HERE / "cuda_vector_search"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["cvs_tc_search.cu", "cvs_tc_pair.cu", "cvs_gemv.cu", "cvs_merge.cu", "cvs_ingest.cu", "cvs_capi.cu"]
LIB_NAME = "libcvs_b200.so"


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA 12.8+ toolkit required)")
    return cand


def _cuda_home() -> Path:
    return Path(_nvcc()).resolve().parent.parent


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}{res.stderr}")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            jobs.append([nvcc] + flags + ["-c", str(s), "-o", str(o)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    lib = PKG / LIB_NAME
    if force or jobs or _stale(lib, objs):
        _run([nvcc] + ARCH + ["-shared", "-o", str(lib)] + [str(o) for o in objs], verbose)
    return lib


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = PKG / ("_C" + suffix)
    src = CSRC / "torch_ext.cpp"
    lib = PKG / LIB_NAME
    if not force and not _stale(out, [src, lib] + _headers()):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in cpp_extension.include_paths()] + [
        f"-I{sysconfig.get_paths()['include']}",
        f"-I{_cuda_home() / 'include'}",
        f"-I{INCLUDE}",
    ]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths()]
    cmd = (
        ["g++", "-O2", "-shared", "-fPIC", "-std=c++17", "-w", str(src), "-o", str(out)]
        + inc
        + ["-DTORCH_EXTENSION_NAME=_C", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
        + libdirs
        + [f"-L{PKG}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN"]
        + ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    )
    _run(cmd, verbose)
    return out


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_torch_ext(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    build(args.force, args.verbose)
    print("built", PKG / LIB_NAME, "and the torch binding", file=sys.stderr)
