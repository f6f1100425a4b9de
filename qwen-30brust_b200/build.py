"""Build recipes for the native libraries (in place, next to this file).

libqwen_cuda.so   sm_100a kernels + host engine + C ABI (include/qwen_cuda.h)
libqwen_tools.so  host-only quantizers and synthetic GGUF writer (include/qwen_tools.h)

`python qwen-30brust_b200/build.py [--verbose-ptxas]` or `build()` from Python.
Objects are rebuilt only when a source or header is newer than the output.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ = HERE / "_build"
CUDA_LIB = HERE / "libqwen_cuda.so"
TOOLS_LIB = HERE / "libqwen_tools.so"

CU_SOURCES = ["matvec.cu", "decode.cu", "token.cu", "engine.cu", "noalloc.cu", "sample.cu", "moe.cu", "batch.cu",
              "qgemm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _cxx() -> str:
    # /usr/bin/g++ first: the image's /opt/gcc wrapper lacks some runtime specs
    for cand in ("/usr/bin/g++", shutil.which("g++"), os.environ.get("CXX")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("g++ not found")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _run(cmd: list[str]) -> str:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build_cuda(verbose_ptxas: bool = False, force: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    nvcc = _nvcc()
    hdrs = _headers()
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
                    "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        flags += ["-Xptxas", "-v"]
    jobs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = OBJ / (src + ".o")
        if force or verbose_ptxas or _stale(o, [s] + hdrs):
            jobs.append([nvcc, *flags, "-c", str(s), "-o", str(o)])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        for out in ex.map(_run, jobs):
            logs.append(out)
    objs = [OBJ / (s + ".o") for s in CU_SOURCES]
    if force or jobs or _stale(CUDA_LIB, objs):
        tmp = CUDA_LIB.with_suffix(".so.tmp")
        _run([nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"])
        os.replace(tmp, CUDA_LIB)
    if verbose_ptxas:
        print("\n".join(logs))
    return CUDA_LIB


def build_tools(force: bool = False) -> Path:
    src = CSRC / "synth.cpp"
    if force or _stale(TOOLS_LIB, [src] + _headers()):
        tmp = TOOLS_LIB.with_suffix(".so.tmp")
        _run([_cxx(), "-O3", "-std=c++17", "-fPIC", "-pthread", "-shared", "-Wall", "-Wextra", "-o", str(tmp), str(src)])
        os.replace(tmp, TOOLS_LIB)
    return TOOLS_LIB


def build(verbose_ptxas: bool = False, force: bool = False) -> None:
    build_tools(force)
    build_cuda(verbose_ptxas, force)


if __name__ == "__main__":
    build(verbose_ptxas="--verbose-ptxas" in sys.argv, force="--force" in sys.argv)
