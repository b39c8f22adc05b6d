"""Batches of bitmaps (the reference's v2 API): layout and input checks on
the CPU, and on the GPU membership, decompress, promotion and multi_and
against numpy truth, for batches built from portable serializations."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]


def test_batch_layout_matches_cpp(tmp_path, built_lib):
    """offsetof() of every field: cr_roaring_batch == cu_roaring::v2::GpuRoaringBatch == ctypes."""
    import cu_roaring_b200 as cr

    fields = [f[0] for f in cr.CrRoaringBatch._fields_]
    body = "\n".join(f'  printf("%s %zu %zu\\n", "{f}", offsetof(cr_roaring_batch, {f}), '
                     f"offsetof(cu_roaring::v2::GpuRoaringBatch, {f}));" for f in fields)
    src = tmp_path / "layout.cpp"
    src.write_text(f"""#include <cstdio>
#include <cstddef>
#include "cu_roaring_b200.h"
#include "cu_roaring_v2/types.cuh"
int main() {{
{body}
  printf("size %zu %zu\\n", sizeof(cr_roaring_batch), sizeof(cu_roaring::v2::GpuRoaringBatch));
}}
""")
    exe = tmp_path / "layout"
    subprocess.run(["g++", "-std=c++17", f"-I{REPO / 'include'}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {line.split()[0]: tuple(map(int, line.split()[1:])) for line in out if line.strip()}
    for f in fields:
        assert got[f][0] == got[f][1] == getattr(cr.CrRoaringBatch, f).offset, f
    assert got["size"][0] == got["size"][1] == C.sizeof(cr.CrRoaringBatch)


def test_batch_rejects_malformed_input(built_lib, oracle):
    """Every buffer is checked before any device work."""
    import cu_roaring_b200 as cr

    good = oracle.serialize_portable([1, 2, 3])
    with pytest.raises(RuntimeError, match="cookie"):
        cr.batch_upload_portable([good, b"\x01\x02\x03\x04" + good[4:]])
    with pytest.raises(RuntimeError, match="truncated"):
        cr.batch_upload_portable([good[:9]])
    # One RUN container holding two overlapping runs (10..19 and 15..24) that
    # declare 20 members: sorted-and-disjoint check.
    bad = bytes.fromhex("3b300000" "01" "00001300" "0200" "0a000900" "0f000900")
    with pytest.raises(RuntimeError, match="disjoint"):
        cr.batch_upload_portable([bad])


def _sets(rng):
    U = 1 << 21
    mixed = []
    for chunk in range(U >> 16):
        base = chunk << 16
        if chunk % 3 == 0:
            mixed.append(base + rng.choice(65536, 500, replace=False))
        elif chunk % 3 == 1:
            mixed.append(base + np.flatnonzero(rng.random(65536) < 0.3))
        else:
            mixed.append(base + np.arange(100, 30000))
    return [np.unique(np.concatenate(mixed)).astype(np.uint32),
            np.flatnonzero(rng.random(U) < 0.01).astype(np.uint32),
            np.array([], dtype=np.uint32),
            np.arange(0, 65536, dtype=np.uint32),  # one full container (cardinality stored as 0)
            np.flatnonzero(rng.random(U // 2) < 0.7).astype(np.uint32)]


def _truth_words(ids, words_each):
    w = np.zeros(words_each * 2, dtype=np.uint32)
    np.bitwise_or.at(w, ids // 32, (np.uint32(1) << (ids % 32)).astype(np.uint32))
    return w.view(np.int64)


@pytest.mark.gpu
def test_batch_queries_decompress_promote_and(cr, oracle):
    import torch

    rng = np.random.default_rng(3)
    sets = _sets(rng)
    batch = cr.batch_upload_portable([oracle.serialize_portable(s) for s in sets])
    assert batch.n_bitmaps == len(sets)
    for b, s in enumerate(sets):
        assert batch.total_cardinality(b) == s.size
        assert batch.universe_size(b) == (0 if s.size == 0 else ((int(s.max()) >> 16) + 1) << 16)
    assert batch.raw.n_bitmap_containers_total < batch.raw.total_containers  # arrays and runs kept

    words_each = (1 << 21) // 64
    truth = [_truth_words(s, words_each) for s in sets]

    def check(bt, what):
        got = bt.decompress(words_each).cpu().numpy()
        for b in range(len(sets)):
            assert np.array_equal(got[b], truth[b]), f"{what}: decompress bitmap {b}"
        n = 1 << 18
        bidx = rng.integers(0, len(sets) + 1, n).astype(np.int32)  # includes an out-of-range bitmap
        ids = np.where(rng.random(n) < 0.5, rng.integers(0, 1 << 21, n),
                       np.concatenate(sets)[rng.integers(0, sum(s.size for s in sets), n)]).astype(np.int32)
        hit = bt.contains(torch.from_numpy(bidx).cuda(), torch.from_numpy(ids).cuda()).cpu().numpy()
        want = np.array([b < len(sets) and (int(i) >> 6) < words_each and
                         bool((truth[b][int(i) >> 6] >> (int(i) & 63)) & 1) for b, i in zip(bidx, ids)])
        assert np.array_equal(hit, want), f"{what}: contains"

    check(batch, "as uploaded")
    prom = batch.promote()
    assert prom.raw.n_bitmap_containers_total == prom.raw.total_containers == batch.raw.total_containers
    check(prom, "promoted")
    with pytest.raises(RuntimeError, match="all-BITMAP"):
        batch.multi_and([0, 1])
    for idx in ([0, 1, 4], [0, 4], [3], [0, 2]):
        r = prom.multi_and(idx)
        want = truth[idx[0]].copy()
        for j in idx[1:]:
            want &= truth[j]
        got = r.decompress(words_each).cpu().numpy()[0]
        assert np.array_equal(got, want), idx
        assert r.total_cardinality(0) == int(np.unpackbits(want.view(np.uint8)).sum())
        r.free()
    prom.free()
    batch.free()
    empty = cr.batch_upload_portable([])
    assert empty.n_bitmaps == 0
    empty.free()
