"""CPU: the C-ABI library builds, loads and exports every symbol that
include/cu_roaring_b200.h declares; the ctypes and C struct layouts agree
with the C++ GpuRoaring layout. No compute calls (no GPU here)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    text = (REPO / "include" / "cu_roaring_b200.h").read_text()
    return set(re.findall(r"\b(cr_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol(built_lib):
    lib = C.CDLL(str(built_lib))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, f"missing exports: {missing}"
    assert len(declared_symbols()) >= 24


def test_python_binding_covers_header(built_lib):
    import cu_roaring_b200 as cr

    assert set(cr.EXPORTED_SYMBOLS) == declared_symbols()
    assert "sm_100a" in cr.version()


def test_struct_layout_matches_cpp(tmp_path, built_lib):
    """offsetof() of every field: C ABI struct == C++ GpuRoaring == ctypes."""
    import cu_roaring_b200 as cr

    src = tmp_path / "layout.cu"
    fields = [f[0] for f in cr.CrGpuRoaring._fields_]
    body = "\n".join(
        f'  printf("%s %zu %zu\\n", "{f}", offsetof(cr_gpu_roaring, {f}), '
        f"offsetof(cu_roaring::GpuRoaring, {f}));" for f in fields)
    src.write_text(f"""#include <cstdio>
#include <cstddef>
#include "cu_roaring_b200.h"
#include "cu_roaring/types.cuh"
int main() {{
{body}
  printf("size %zu %zu\\n", sizeof(cr_gpu_roaring), sizeof(cu_roaring::GpuRoaring));
}}
""")
    exe = tmp_path / "layout"
    subprocess.run(["g++", "-x", "c++", "-std=c++17", f"-I{REPO / 'include'}", str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {line.split()[0]: tuple(map(int, line.split()[1:])) for line in out if line.strip()}
    for f in fields:
        c_off, cpp_off = got[f]
        assert c_off == cpp_off == getattr(cr.CrGpuRoaring, f).offset, f
    assert got["size"][0] == got["size"][1] == C.sizeof(cr.CrGpuRoaring)


def test_error_path_without_gpu(built_lib):
    """Argument validation runs before any device work: a null output
    pointer returns CR_ERR_INVALID with a message, even without a GPU."""
    import cu_roaring_b200 as cr

    rc = cr.lib().cr_set_operation(None, None, 0, None, None)
    assert rc == -1
    assert b"null" in cr.lib().cr_last_error_string()


def _layout_program(tmp_path, include_dir: Path, tag: str) -> str:
    """Compiles and runs a host program printing sizeof / offsetof of every
    field of GpuRoaring, GpuRoaringMeta and GpuRoaringView as declared by the
    headers under include_dir."""
    roaring = ["keys", "types", "offsets", "cardinalities", "n_containers", "universe_size", "total_cardinality",
               "bitmap_data", "n_bitmap_containers", "array_data", "n_array_containers", "array_pool_bytes",
               "run_data", "n_run_containers", "run_pool_bytes", "key_index", "max_key", "negated", "_alloc_base"]
    meta = ["n_containers", "n_bitmap_containers", "n_array_containers", "n_run_containers", "universe_size",
            "total_bytes"]
    view = ["keys", "types", "offsets", "cardinalities", "n_containers", "bitmap_data", "array_data", "run_data",
            "key_index", "max_key", "all_bitmap", "negated"]
    lines = []
    for struct, fields in (("GpuRoaring", roaring), ("GpuRoaringMeta", meta), ("GpuRoaringView", view)):
        lines.append(f'  printf("{struct} size %zu\\n", sizeof(cu_roaring::{struct}));')
        for f in fields:
            lines.append(f'  printf("{struct}.{f} %zu\\n", offsetof(cu_roaring::{struct}, {f}));')
    src = tmp_path / f"layout_{tag}.cu"
    src.write_text("#include <cstddef>\n#include <cstdio>\n#include \"cu_roaring/types.cuh\"\n"
                   "#include \"cu_roaring/device/roaring_view.cuh\"\nint main() {\n" + "\n".join(lines) +
                   "\n  return 0;\n}\n")
    exe = tmp_path / f"layout_{tag}"
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-std=c++17", f"-I{include_dir}", str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout


def test_layouts_match_the_reference_headers(tmp_path):
    """The public structs (GpuRoaring, GpuRoaringMeta, GpuRoaringView) have the
    reference's exact layout: the reference's own include/cu_roaring headers
    and this engine's, compiled side by side. Runs where the reference
    checkout is present (CU_ROARING_REFERENCE, default /root/reference)."""
    import os

    ref = Path(os.environ.get("CU_ROARING_REFERENCE", "/root/reference")) / "include"
    if not (ref / "cu_roaring" / "types.cuh").exists():
        import pytest

        pytest.skip("reference headers not present")
    ours = _layout_program(tmp_path, REPO / "include", "ours")
    theirs = _layout_program(tmp_path, ref, "ref")
    assert ours == theirs
