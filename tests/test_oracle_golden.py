"""CPU: the oracle against the known answers of the reference's own tests.

Each case cites the reference test it replays. Truth is computed directly
from the ID lists with numpy, independently of any Roaring structure.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import ref_sets

KEEP, ALL, AUTO = 4096, 0, 0xFFFFFFFF
AND, OR, ANDNOT, XOR = 0, 1, 2, 3


def truth_words(ids, universe):
    w = np.zeros((universe + 31) // 32, dtype=np.uint32)
    ids = np.unique(np.asarray(ids, dtype=np.uint64))
    np.bitwise_or.at(w, (ids // 32).astype(np.int64), (1 << (ids % 32)).astype(np.uint32))
    return w


def np_op(a, b, op):
    return {AND: a & b, OR: a | b, ANDNOT: a & ~b, XOR: a ^ b}[op]


def forced_negated(oracle, logical_words, universe):
    """A bitmap whose STORED set is the complement of `logical_words` with
    negated=true (test/test_complement.cu:372-397 builds its operands so)."""
    comp = ~logical_words
    tail = universe % 32
    if tail:
        comp[-1] &= (1 << tail) - 1
    big = universe * 4  # large universe: no automatic complement
    b = oracle.from_bitset(comp, big, KEEP)
    b.im.negated = 1
    b.im.universe_size = universe
    b.im.total_cardinality = int(np.unpackbits(logical_words.view(np.uint8)).sum())
    return b


# ---- test/test_promote.cu:387-449 -----------------------------------------

def test_unsorted_duplicates(oracle):
    b = oracle.from_ids([200, 5, 100000, 42, 65536, 0, 100000, 5], 200000, KEEP)
    assert b.image()["total_cardinality"] == 6
    assert list(b.enumerate()) == [0, 5, 42, 200, 65536, 100000]
    bits = b.contains(np.array([1, 100, 65535], dtype=np.uint32))
    assert bits[0] & 0b111 == 0
    assert b.validate() == 0


def test_all_duplicates(oracle):
    im = oracle.from_ids([42, 42, 42, 42], 100, KEEP).image()
    assert im["total_cardinality"] == 1 and im["n_containers"] == 1


def test_reversed(oracle):
    b = oracle.from_ids(np.arange(999, -1, -1), 1000, KEEP)
    im = b.image()
    assert im["total_cardinality"] == 1000
    assert im["negated"]  # 1000 > 1000/2: stored as the (empty) complement
    assert np.unpackbits(b.decompress().view(np.uint8)).sum() == 1000


def test_threshold_counts(oracle):  # test/test_promote.cu:183-216
    ids = np.array([k * 65536 + j * 100 for k in range(5) for j in range(100)], dtype=np.uint32)
    arr = oracle.from_ids(ids, 5 * 65536, KEEP).image()
    assert (arr["n_containers"], arr["n_array"], arr["n_bitmap"]) == (5, 5, 0)
    bmp = oracle.from_ids(ids, 5 * 65536, ALL).image()
    assert (bmp["n_containers"], bmp["n_bitmap"], bmp["n_array"]) == (5, 5, 0)


def test_custom_threshold(oracle):  # test/test_promote.cu:218-251
    ids = np.array([k * 65536 + j for k in range(3) for j in range(200)], dtype=np.uint32)
    bmp = oracle.from_ids(ids, 3 * 65536, 100).image()
    assert (bmp["n_bitmap"], bmp["n_array"]) == (3, 0)
    arr = oracle.from_ids(ids, 3 * 65536, KEEP).image()
    assert (arr["n_array"], arr["n_bitmap"]) == (3, 0)


def test_auto_resolution(oracle):  # test/test_promote.cu:257-267
    assert oracle.resolve_auto_threshold(1_000_000) == KEEP
    assert oracle.resolve_auto_threshold(1_000_000_000) == ALL


# ---- test/test_complement.cu ----------------------------------------------

def test_negated_small(oracle):  # :129-150
    ids = [0, 1, 2, 3, 4, 5, 6, 8, 9]
    b = oracle.from_ids(ids, 10)
    assert b.image()["negated"]
    bits = b.contains(np.arange(10, dtype=np.uint32))[0]
    assert [(bits >> i) & 1 for i in range(10)] == [1, 1, 1, 1, 1, 1, 1, 0, 1, 1]


@pytest.mark.parametrize("name,neg", [("compl_absent_key", True), ("compl_large", True),
                                      ("compl_low", False)])
def test_complement_flags(oracle, name, neg):  # :151-225
    words, u = ref_sets.load(name)
    b = oracle.from_ids(ref_sets.ids_of(words), u)
    assert b.image()["negated"] == neg
    assert np.array_equal(b.decompress(), words)
    assert b.validate() == 0
    q = np.arange(0, u, 7, dtype=np.uint32)
    got = np.unpackbits(b.contains(q).view(np.uint8), bitorder="little")[: q.size]
    want = (words[q // 32] >> (q % 32)) & 1
    assert np.array_equal(got, want)


def test_exactly_half_not_negated(oracle):  # :227-241
    assert not oracle.from_ids(np.arange(50), 100).image()["negated"]


def test_user_example(oracle):  # :320-353  NOT{7} AND {4,6,7} = {4,6}
    a = oracle.from_ids([0, 1, 2, 3, 4, 5, 6, 8, 9], 10)
    assert a.image()["negated"]
    b = oracle.from_ids([4, 6, 7], 10)
    r = oracle.set_operation(a, b, AND)
    assert list(r.enumerate()) == [4, 6]


@pytest.mark.parametrize("op", [AND, OR, ANDNOT, XOR])
@pytest.mark.parametrize("na,nb", [(False, False), (True, False), (False, True), (True, True)])
def test_demorgan(oracle, op, na, nb):  # :441-462 all 16 combinations
    wa, u = ref_sets.load("demorgan_a")
    wb, _ = ref_sets.load("demorgan_b")
    a = forced_negated(oracle, wa, u) if na else oracle.from_bitset(wa, u, KEEP)
    b = forced_negated(oracle, wb, u) if nb else oracle.from_bitset(wb, u, KEEP)
    r = oracle.set_operation(a, b, op)
    assert np.array_equal(r.decompress((u + 31) // 32), np_op(wa, wb, op))
    assert r.validate() == 0


SETOPS = [("setops_bb_a", "setops_bb_b", AND), ("setops_aa_a", "setops_aa_b", AND),
          ("setops_ba_a", "setops_ba_b", AND), ("setops_disjoint_a", "setops_disjoint_b", AND),
          ("setops_ident", "setops_ident", AND), ("setops_or_a", "setops_or_b", OR),
          ("setops_disjoint_a", "setops_disjoint_b", OR),
          ("setops_andnot_a", "setops_andnot_b", ANDNOT), ("setops_xor_a", "setops_xor_b", XOR),
          ("setops_xor_ident", "setops_xor_ident", XOR)]


@pytest.mark.parametrize("an,bn,op", SETOPS)
@pytest.mark.parametrize("thr", [KEEP, ALL])
def test_setops(oracle, an, bn, op, thr):  # test/test_set_ops.cu:84-288
    wa, u = ref_sets.load(an)
    wb, _ = ref_sets.load(bn)
    a, b = oracle.from_bitset(wa, u, thr), oracle.from_bitset(wb, u, thr)
    r = oracle.set_operation(a, b, op)
    want = np_op(wa, wb, op)
    assert np.array_equal(r.decompress(len(want)), want)
    assert r.validate() == 0
    assert r.image()["total_cardinality"] == int(np.unpackbits(want.view(np.uint8)).sum())


@pytest.mark.parametrize("names,fn", [
    (["setops_mand_a", "setops_mand_b", "setops_mand_c"], "and"),
    (["setops_mor_a", "setops_mor_b", "setops_mor_c"], "or"),
    (["mand_neg_1", "mand_neg_2", "mand_neg_3"], "and"),
    (["mand_allneg_1", "mand_allneg_2", "mand_allneg_3"], "and"),
    (["absent_A", "absent_B", "absent_C"], "and"),
    ([f"mixed5_{i}" for i in range(5)], "and"),
    ([f"alt8_{i}" for i in range(8)], "and"),
    ([f"alt8_{i}" for i in range(8)], "or"),
])
def test_multi(oracle, names, fn):  # test/test_set_ops.cu:290-342, test/test_complement.cu:503-790
    sets = [ref_sets.load(n) for n in names]
    bms = [oracle.from_bitset(w, u, ALL) for w, u in sets]
    r = (oracle.multi_and if fn == "and" else oracle.multi_or)(bms)
    want = sets[0][0].copy()
    for w, _ in sets[1:]:
        want = (want & w) if fn == "and" else (want | w)
    assert np.array_equal(r.decompress(len(want)), want)
    assert r.validate() == 0


def test_mixed_negation_flags(oracle):  # test/test_complement.cu:711-716, :768
    flags = [oracle.from_bitset(*ref_sets.load(f"mixed5_{i}"), ALL).image()["negated"] for i in range(5)]
    assert flags == [False, True, False, True, False]
    flags = [oracle.from_bitset(*ref_sets.load(f"alt8_{i}"), ALL).image()["negated"] for i in range(8)]
    assert flags == [i % 2 == 1 for i in range(8)]


# ---- test/test_decompress.cu, test/test_device_query.cu --------------------

def test_boundary_and_full(oracle):  # test/test_decompress.cu:200-232
    b = oracle.from_ids([65535, 65536], 200000, KEEP)
    assert list(b.enumerate()) == [65535, 65536]
    full = oracle.from_ids(np.arange(65536), 10 * 65536, KEEP)
    im = full.image()
    assert im["n_run"] == 1 and im["run"].tolist() == [0, 65535]
    assert full.enumerate().size == 65536


def test_run_containers(oracle):  # test/test_device_query.cu:153-169
    ids = np.concatenate([np.arange(1000, 5001), np.arange(70000, 80001)])
    b = oracle.from_ids(ids, 200000, KEEP)
    im = b.image()
    assert im["types"].tolist() == [0, 2]  # 4001 <= 4096 -> ARRAY; 10001 -> RUN
    q = np.arange(0, 100000, dtype=np.uint32)
    got = np.unpackbits(b.contains(q).view(np.uint8), bitorder="little")[: q.size]
    assert np.array_equal(np.flatnonzero(got), ids)


def test_container_rule(oracle):
    assert oracle.container_type(100, 100, KEEP) == 0
    assert oracle.container_type(4097, 5000, KEEP) == 1
    assert oracle.container_type(30000, 10, KEEP) == 2
    assert oracle.container_type(65536, 1, ALL) == 1
    assert oracle.container_type(200, 1, 100) == 1
    assert oracle.container_type(5000, 10, 10000) == 2  # 40 B of runs < 10000 B array
    assert oracle.container_type(5000, 3000, 10000) == 0


def test_promote_and_uniform(oracle):
    words, u = ref_sets.load("uniform_int_1e6")
    b = oracle.from_bitset(words, u, KEEP)
    p = oracle.promote_to_bitmap(b)
    assert p.image()["n_bitmap"] == b.image()["n_containers"]
    assert np.array_equal(p.decompress(), words) and p.validate() == 0
