"""Build script for the cu_roaring B200 engine.

Compiles every CUDA source under csrc/ for sm_100a with nvcc (one object per
source, rebuilt only when a source or header is newer), links
cu_roaring_b200/libcuroaring_b200.so in-tree, and builds the C++ drop-in
header test program. `python build.py` or `build_all()`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "cu_roaring_b200" / "libcuroaring_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         f"-I{REPO / 'include'}", f"-I{CSRC}"]


def _headers() -> list[Path]:
    inc = REPO / "include"
    return list(CSRC.glob("*.cuh")) + [p for ext in ("*.h", "*.hpp", "*.cuh") for p in inc.rglob(ext)]


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def build_lib(force: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    hdr_time = _newest(_headers())
    jobs = []
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            # topk.cu launches its exact redo from the device (relocatable device code)
            rdc = ["-rdc=true"] if src.stem == "topk" else []
            jobs.append([NVCC, *ARCH, *FLAGS, *rdc, "-c", str(src), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(_run, jobs))
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < _newest(objs):
        _run([NVCC, *ARCH, "-shared", "-rdc=true", "--cudart", "shared", "-o", str(LIB), *map(str, objs),
              "-lcudadevrt", "-Xlinker", "-rpath,/usr/local/cuda/lib64"])
    return LIB


def build_cpp_tests(force: bool = False) -> Path | None:
    """The C++ drop-in test: user kernels over the public headers, linked to the .so."""
    src = REPO / "tests" / "cpp" / "api_test.cu"
    if not src.exists():
        return None
    out_dir = REPO / "tests" / "cpp" / "_build"
    out_dir.mkdir(parents=True, exist_ok=True)
    exe = out_dir / "api_test"
    if force or not exe.exists() or exe.stat().st_mtime < max(src.stat().st_mtime, _newest(_headers()),
                                                              LIB.stat().st_mtime):
        _run([NVCC, *ARCH, *FLAGS, "--cudart", "shared", str(src), "-o", str(exe),
              f"-L{LIB.parent}", "-lcuroaring_b200",
              "-Xlinker", f"-rpath,{LIB.parent}:/usr/local/cuda/lib64"])
    return exe


def build_all(force: bool = False) -> None:
    build_lib(force)
    build_cpp_tests(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(LIB)
