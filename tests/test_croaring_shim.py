"""The CRoaring-typed upload() / get_meta() overloads of the drop-in headers
(include/cu_roaring/detail/upload.cuh), built against a test-only stub of
CRoaring's public API (tests/cpp/croaring_stub) whose portable serialization
comes from the CPU oracle's writer.

CPU: the guarded block compiles and links. GPU: the program's checks pass."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _build(built_lib) -> Path:
    import oracle

    oracle.build()
    src = REPO / "tests" / "cpp" / "croaring_test.cu"
    out_dir = REPO / "tests" / "cpp" / "_build"
    out_dir.mkdir(parents=True, exist_ok=True)
    exe = out_dir / "croaring_test"
    newest = max(p.stat().st_mtime for p in [src, Path(built_lib), REPO / "include" / "cu_roaring" / "detail" /
                                              "upload.cuh", REPO / "tests" / "cpp" / "croaring_stub" / "roaring" /
                                              "roaring.h"])
    if not exe.exists() or exe.stat().st_mtime < newest:
        cmd = ["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
               f"-I{REPO / 'include'}", f"-I{REPO / 'tests' / 'cpp' / 'croaring_stub'}", str(src), "-o", str(exe),
               "--cudart", "shared", f"-L{Path(built_lib).parent}", "-lcuroaring_b200", f"-L{REPO / 'oracle'}",
               "-loracle", "-Xlinker", f"-rpath,{Path(built_lib).parent}:{REPO / 'oracle'}:/usr/local/cuda/lib64"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        assert res.returncode == 0, res.stdout + res.stderr
    return exe


def test_croaring_overloads_compile(built_lib):
    assert _build(built_lib).exists()


@pytest.mark.gpu
def test_croaring_overloads_run(built_lib, cr):
    res = subprocess.run([str(_build(built_lib))], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert " 0 failed" in res.stdout
