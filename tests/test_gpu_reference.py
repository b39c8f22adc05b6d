"""GPU: this engine against the REFERENCE's own CUDA implementation.

oracle/_ref/libref_cu_roaring.so is the reference's src/upload_ids.cu,
promote.cu, set_ops.cu, decompress.cu and to_csr.cu compiled unmodified for
sm_100a (oracle/build_ref.py). The same inputs go through both; the logical
results (decompressed bitsets, sorted IDs, cardinalities, negation flags)
must be identical. Container layouts legitimately differ (the reference's GPU
path is all-BITMAP; this engine selects ARRAY/BITMAP/RUN), so layouts are
compared against the CPU oracle elsewhere and only the sets here.

Also checks the drop-in direction: this engine's kernels (contains,
enumerate, set operations) consume bitmaps BUILT BY THE REFERENCE.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import ref_sets

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_cu_roaring.so"


@pytest.fixture(scope="module")
def ref(cr):
    if not REF_LIB.exists():
        pytest.skip("reference library not built (oracle/build_ref.py needs the reference sources)")
    lib = C.CDLL(str(REF_LIB))
    P = C.POINTER(cr.CrGpuRoaring)
    sig = {
        "ref_upload_from_ids": ([C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, P], C.c_int),
        "ref_upload_from_bitset": ([C.c_void_p, C.c_uint32, C.c_uint32, P], C.c_int),
        "ref_set_operation": ([P, P, C.c_int, P], C.c_int),
        "ref_multi_and": ([P, C.c_uint32, P], C.c_int),
        "ref_multi_or": ([P, C.c_uint32, P], C.c_int),
        "ref_decompress": ([P, C.c_void_p, C.c_uint32], C.c_int),
        "ref_enumerate": ([P, C.c_void_p], C.c_int),
        "ref_free": ([P], C.c_int),
        "ref_last_error": ([], C.c_char_p),
        "ref_resolve_auto_threshold": ([C.c_uint32], C.c_uint32),
    }
    for n, (a, r) in sig.items():
        f = getattr(lib, n)
        f.argtypes = a
        f.restype = r
    return lib


def ref_call(ref, fn, *args):
    rc = getattr(ref, fn)(*args)
    assert rc == 0, f"{fn}: {ref.ref_last_error().decode()}"


def ref_upload_ids(ref, cr, ids, u, thr=0xFFFFFFFF):
    out = cr.CrGpuRoaring()
    a = np.ascontiguousarray(ids, dtype=np.uint32)
    ref_call(ref, "ref_upload_from_ids", a.ctypes.data, a.size, u, thr, C.byref(out))
    return out


def ref_bits(ref, raw, u):
    w = np.zeros((u + 31) // 32, dtype=np.uint32)
    ref_call(ref, "ref_decompress", C.byref(raw), w.ctypes.data, w.size)
    return w


def our_bits(cr, bm, u):
    import torch

    out = torch.zeros(((u + 31) // 32,), dtype=torch.int32, device="cuda")
    return cr.decompress_to_bitset(bm, output=out).cpu().numpy().view(np.uint32)


NAMES = ["setops_bb_a", "setops_aa_a", "compl_absent_key", "compl_low", "absent_B", "mixed5_1",
         "uniform_int_1e6"]


@pytest.mark.parametrize("name", NAMES)
def test_upload_from_ids_same_set_as_reference(cr, ref, name):
    words, u = ref_sets.load(name)
    ids = ref_sets.ids_of(words)
    rng = np.random.default_rng(1)
    ids = np.concatenate([ids, ids[: ids.size // 20]])
    rng.shuffle(ids)
    r = ref_upload_ids(ref, cr, ids, u)
    ours = cr.upload_from_ids(ids, u)
    assert bool(r.negated) == bool(ours.raw.negated)
    assert r.total_cardinality == ours.raw.total_cardinality
    assert np.array_equal(ref_bits(ref, r, u), our_bits(cr, ours, u))
    assert np.array_equal(ref_bits(ref, r, u), words)
    ref_call(ref, "ref_free", C.byref(r))
    ours.free()


@pytest.mark.parametrize("name", NAMES[:5])
def test_upload_from_bitset_same_set_as_reference(cr, ref, name):
    words, u = ref_sets.load(name)
    r = cr.CrGpuRoaring()
    ref_call(ref, "ref_upload_from_bitset", words.ctypes.data, words.size, u, C.byref(r))
    ours = cr.upload_from_bitset(words, u)
    assert bool(r.negated) == bool(ours.raw.negated)
    assert r.total_cardinality == ours.raw.total_cardinality
    assert np.array_equal(ref_bits(ref, r, u), our_bits(cr, ours, u))
    ref_call(ref, "ref_free", C.byref(r))
    ours.free()


PAIRS = [("setops_bb_a", "setops_bb_b"), ("setops_aa_a", "setops_aa_b"), ("setops_ba_a", "setops_ba_b"),
         ("demorgan_a", "demorgan_b"), ("compl_absent_key", "setops_bb_b")]


@pytest.mark.parametrize("an,bn", PAIRS)
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_set_operation_same_set_as_reference(cr, ref, an, bn, op):
    wa, ua = ref_sets.load(an)
    wb, ub = ref_sets.load(bn)
    u = max(ua, ub)
    ia, ib = ref_sets.ids_of(wa), ref_sets.ids_of(wb)
    ra, rb = ref_upload_ids(ref, cr, ia, u), ref_upload_ids(ref, cr, ib, u)
    oa, ob = cr.upload_from_ids(ia, u), cr.upload_from_ids(ib, u)
    rr = cr.CrGpuRoaring()
    ref_call(ref, "ref_set_operation", C.byref(ra), C.byref(rb), op, C.byref(rr))
    orr = cr.set_operation(oa, ob, op)
    assert np.array_equal(ref_bits(ref, rr, u), our_bits(cr, orr, u))
    # drop-in direction: this engine's set operation on the reference's own bitmaps
    cross = cr.set_operation(cr.GpuRoaring(ra), cr.GpuRoaring(rb), op)
    assert np.array_equal(ref_bits(ref, rr, u), our_bits(cr, cross, u))
    for x in (ra, rb, rr):
        ref_call(ref, "ref_free", C.byref(x))
    for x in (oa, ob, orr, cross):
        x.free()


@pytest.mark.parametrize("names,fn", [
    (["setops_mand_a", "setops_mand_b", "setops_mand_c"], "and"),
    (["mand_neg_1", "mand_neg_2", "mand_neg_3"], "and"),
    ([f"mixed5_{i}" for i in range(5)], "and"),
    ([f"alt8_{i}" for i in range(8)], "and"),
    (["setops_mor_a", "setops_mor_b", "setops_mor_c"], "or"),
])
def test_multi_same_set_as_reference(cr, ref, names, fn):
    sets = [ref_sets.load(n) for n in names]
    u = max(x[1] for x in sets)
    refs = (cr.CrGpuRoaring * len(sets))()
    ours = []
    for i, (w, _) in enumerate(sets):
        refs[i] = ref_upload_ids(ref, cr, ref_sets.ids_of(w), u, 0)
        ours.append(cr.upload_from_ids(ref_sets.ids_of(w), u, bitmap_threshold=0))
    rr = cr.CrGpuRoaring()
    ref_call(ref, "ref_multi_and" if fn == "and" else "ref_multi_or", refs, len(sets), C.byref(rr))
    orr = (cr.multi_and if fn == "and" else cr.multi_or)(ours)
    assert np.array_equal(ref_bits(ref, rr, u), our_bits(cr, orr, u))
    for i in range(len(sets)):
        ref_call(ref, "ref_free", C.byref(refs[i]))
    ref_call(ref, "ref_free", C.byref(rr))
    for x in ours + [orr]:
        x.free()


@pytest.mark.parametrize("name", ["setops_bb_a", "setops_aa_a", "compl_low", "uniform_int_1e6"])
def test_enumerate_and_contains_on_reference_bitmaps(cr, ref, name):
    import torch

    words, u = ref_sets.load(name)
    ids = ref_sets.ids_of(words)
    r = ref_upload_ids(ref, cr, ids, u)
    rb = cr.GpuRoaring(r)
    if not r.negated:  # the reference's enumerate_ids ignores `negated`
        got = np.zeros(max(1, r.total_cardinality), dtype=np.int64)
        ref_call(ref, "ref_enumerate", C.byref(r), got.ctypes.data)
        assert np.array_equal(got[: r.total_cardinality], ids.astype(np.int64))
    assert np.array_equal(cr.enumerate_ids(rb).cpu().numpy(), ids.astype(np.int64))
    q = np.random.default_rng(3).integers(0, u, 100_000, dtype=np.uint64).astype(np.uint32)
    dq = torch.from_numpy(q.view(np.int32)).cuda()
    want = ((words[q // 32] >> (q % 32)) & 1).astype(bool)
    for warp in (False, True):
        bits = cr.contains_batch(rb, dq, warp=warp).cpu().numpy().view(np.uint32)
        got = np.unpackbits(bits.view(np.uint8), bitorder="little")[: q.size].astype(bool)
        assert np.array_equal(got, want)
    ref_call(ref, "ref_free", C.byref(r))


def test_auto_threshold_agrees(cr, ref):
    for u in (1_000_000, 1 << 24, 1_000_000_000, 1 << 30, 0xFFFFFFFF):
        assert ref.ref_resolve_auto_threshold(u) == cr.resolve_auto_threshold(u)
