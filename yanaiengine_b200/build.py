"""Build recipe for libyk.so (the sm_100a CUDA module behind include/yk.h).

Compiles every csrc/*.cu with nvcc for sm_100a only and links one shared
library in-tree (yanaiengine_b200/libyk.so), with the CUDA runtime linked
statically so the library loads on a box without a matching libcudart.
The driver API (cuTensorMapEncodeTiled) is resolved at run time through
cudaGetDriverEntryPoint, so no -lcuda is needed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libyk.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libyk.so")
    return cand


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [PKG.parent / "include" / "yk.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps if d.exists()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


HOST_SRC = PKG / "host" / "yk_host.cpp"
HOST_LIB = PKG / "libyk_host.so"


def build_host() -> Path:
    """libyk_host.so: the C++ Scheduler host, linked against libyk.so (rpath $ORIGIN)."""
    lib = build()
    deps = [HOST_SRC, PKG.parent / "include" / "yk_host.h", PKG.parent / "include" / "yk.h", lib]
    if HOST_LIB.exists() and all(HOST_LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return HOST_LIB
    cxx = shutil.which("g++") or "g++"
    tmp = HOST_LIB.with_suffix(".so.tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-o", str(tmp), str(HOST_SRC),
           f"-L{PKG}", "-l:libyk.so", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host library build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, HOST_LIB)
    return HOST_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_host())
