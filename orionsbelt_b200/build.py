"""Build libkai_gdn_cuda.so from orionsbelt_b200/csrc/*.cu for sm_100a.

Plain nvcc, no torch extension machinery: the product is a C-ABI shared
library (include/kai_gdn_cuda.h) with the CUDA runtime linked statically, so
it loads into any host process (C, Python ctypes, ...).  Objects go to
orionsbelt_b200/_build/ and are rebuilt when their source or a header changes.

    python -m orionsbelt_b200.build [-v] [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libkai_gdn_cuda.so"
SELFTEST_SRC = ROOT / "tests" / "c" / "umma_selftest.cu"
SELFTEST_LIB = ROOT / "tests" / "c" / "bin" / "libumma_selftest.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3", "-I", str(ROOT / "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, flush=True)


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda so: _compile(so[0], so[1], verbose), jobs))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def build_selftest(verbose: bool = False) -> Path:
    """Test-only library checking the tcgen05 building blocks (tests/c/umma_selftest.cu)."""
    SELFTEST_LIB.parent.mkdir(parents=True, exist_ok=True)
    deps = [SELFTEST_SRC, CSRC / "umma.cuh", CSRC / "tma.cuh"]
    if SELFTEST_LIB.exists() and SELFTEST_LIB.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return SELFTEST_LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-shared", "-cudart", "static", str(SELFTEST_SRC), "-o", str(SELFTEST_LIB)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {SELFTEST_SRC.name}:\n{r.stdout}\n{r.stderr}")
    return SELFTEST_LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    build_selftest(verbose="-v" in sys.argv)
    print(LIB)
