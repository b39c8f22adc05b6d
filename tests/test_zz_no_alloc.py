"""GPU: the allocation-free enumerate entry point against the regular one.

cr_enumerate_ids_u32_noalloc exists for callers that cannot allocate device
memory while they run (a server whose memory is all handed to its own pool,
or a path where an allocator call is not allowed); it keeps its scratch in a
fixed array inside the library. Here it is called through the C ABI twice in
a row on each bitmap (the second call reuses the array the first one left
behind) and must return exactly what cr_enumerate_ids_u32 returns. This file
is collected last so that a stop-at-first-failure run has already run every
other test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import ref_sets

pytestmark = pytest.mark.gpu


def noalloc(cr, bm, out):
    return cr.lib().cr_enumerate_ids_u32_noalloc(C.byref(bm.raw), out.data_ptr(), None)


@pytest.mark.parametrize("name,thr", [("setops_bb_a", 4096), ("setops_aa_a", 4096), ("compl_absent_key", 4096),
                                      ("absent_B", 0), ("uniform_int_1e6", 4096), ("alt8_1", 0)])
def test_noalloc_matches_regular_twice(cr, name, thr):
    import torch

    words, u = ref_sets.load(name)
    bm = cr.upload_from_bitset(words, u, bitmap_threshold=thr)
    want = cr.enumerate_ids(bm, dtype="uint32").cpu().numpy().view(np.uint32)
    assert want.size == bm.raw.total_cardinality
    for _ in range(2):
        out = torch.full((max(1, want.size),), -1, dtype=torch.int32, device="cuda")
        rc = noalloc(cr, bm, out)
        assert rc == 0, cr.lib().cr_last_error_string()
        torch.cuda.synchronize()
        assert np.array_equal(out[: want.size].cpu().numpy().view(np.uint32), want)
    bm.free()


def test_noalloc_without_key_index(cr):
    """A bitmap assembled elsewhere without key_index: the index is built in
    the fixed scratch, twice in a row."""
    import torch

    words, u = ref_sets.load("compl_large")  # negated: the lookup path is used
    bm = cr.upload_from_bitset(words, u)
    assert bm.raw.negated
    want = cr.enumerate_ids(bm, dtype="uint32").cpu().numpy().view(np.uint32)
    stripped = cr.GpuRoaring(cr.CrGpuRoaring.from_buffer_copy(bm.raw))
    stripped.raw.key_index = None
    for _ in range(2):
        out = torch.zeros((want.size,), dtype=torch.int32, device="cuda")
        assert noalloc(cr, stripped, out) == 0, cr.lib().cr_last_error_string()
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want)
    bm.free()


def test_noalloc_rejects_oversized(cr):
    import torch

    fake = cr.GpuRoaring()
    fake.raw.n_containers = 70000
    fake.raw.total_cardinality = 1
    fake.raw.universe_size = 1 << 31
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = noalloc(cr, fake, out)
    assert rc == -1
    assert b"65536" in cr.lib().cr_last_error_string()
