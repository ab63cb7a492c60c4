"""Builds libgollama_cuda.so in-tree with nvcc for sm_100a.

Every .cu/.cpp file under gollama_b200/csrc is compiled to an object under
gollama_b200/_build (incrementally: a source is rebuilt when it or any header
in csrc/ or include/ is newer than its object) and linked into
gollama_b200/libgollama_cuda.so.  The CUDA runtime is linked statically; NCCL
is resolved at run time with dlopen.
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
LIB = PKG / "libgollama_cuda.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(INCLUDE),
    "-I", str(CSRC),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgollama_cuda.so")


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if "-v" in extra:
        print(f"== {src.name}\n{r.stderr}")


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if ptxas_info or _stale(src, obj, newest_header):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, extra) for s, o in jobs]
            for f in futs:
                f.result()
    if jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"built {LIB}")
    return LIB


SELFTEST_SRC = ROOT / "tests" / "native" / "selftest.cu"
SELFTEST_LIB = ROOT / "tests" / "native" / "_build" / "libglc_selftest.so"


def build_selftest() -> Path:
    """Test-only kernels (tests/native/selftest.cu) as their own shared object;
    nothing of it is linked into libgollama_cuda.so."""
    if SELFTEST_LIB.exists() and SELFTEST_LIB.stat().st_mtime > max(
            SELFTEST_SRC.stat().st_mtime, (CSRC / "sm100.cuh").stat().st_mtime):
        return SELFTEST_LIB
    SELFTEST_LIB.parent.mkdir(parents=True, exist_ok=True)
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-shared", "-o", str(SELFTEST_LIB), str(SELFTEST_SRC)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {SELFTEST_SRC.name}:\n{r.stdout}\n{r.stderr}")
    return SELFTEST_LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas-info" in sys.argv)
