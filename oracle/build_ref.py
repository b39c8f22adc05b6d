"""Builds oracle/_ref/libref_cu_roaring.so from the reference's own CUDA
sources, compiled unmodified where they lie (nvcc, sm_100a), plus
oracle/ref_shim.cu. TEST INFRASTRUCTURE ONLY (a parity pin, never linked
into the product). The reference's CRoaring-based src/upload.cpp is not
built: CRoaring is absent, so only a forward declaration of its bitmap type
is provided (oracle/_ref/shim/roaring/roaring.h, written by this script) for
the one header (detail/upload.cuh) that names it in signatures."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
# The reference checkout: first argument, else CU_ROARING_REFERENCE, else the
# default location of the read-only checkout.
REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CU_ROARING_REFERENCE", "/root/reference"))
OUT = HERE / "_ref"
LIB = OUT / "libref_cu_roaring.so"
SOURCES = ["src/upload_ids.cu", "src/promote.cu", "src/set_ops.cu", "src/decompress.cu", "src/to_csr.cu"]


def main() -> int:
    if not (REF / "include" / "cu_roaring").exists():
        print("reference not present; skipping oracle/_ref build")
        return 0
    shim = OUT / "shim" / "roaring"
    shim.mkdir(parents=True, exist_ok=True)
    (shim / "roaring.h").write_text(
        "/* forward declaration only: CRoaring is absent in this build */\n"
        "#pragma once\ntypedef struct roaring_bitmap_s roaring_bitmap_t;\n")
    srcs = [REF / s for s in SOURCES] + [HERE / "ref_shim.cu"]
    newest = max(p.stat().st_mtime for p in srcs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return 0
    cmd = ["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2",
           "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "--cudart", "shared",
           f"-I{REF / 'include'}", f"-I{OUT / 'shim'}", "-o", str(LIB), *map(str, srcs),
           "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        print(res.stdout, res.stderr, file=sys.stderr)
        return res.returncode
    print(LIB)
    return 0


if __name__ == "__main__":
    sys.exit(main())
