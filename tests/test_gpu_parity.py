"""GPU parity: the sm_100a engine (through the C ABI) against the CPU oracle.

Every comparison is bit-exact: the full packed image (keys, types, offsets,
cardinality fields, key_index, the three pools, counts and flags), the
logical bitset, the sorted IDs and the contains bits. Inputs are the
reference test suite's own sets (tests/golden) plus seeded synthetic data in
the shapes of BASELINE config 1 at reduced size.
"""
from __future__ import annotations

import numpy as np
import pytest

import ref_sets

pytestmark = pytest.mark.gpu

KEEP, ALL, AUTO = 4096, 0, 0xFFFFFFFF
AND, OR, ANDNOT, XOR = 0, 1, 2, 3


@pytest.fixture(scope="module")
def torch_():
    import torch

    return torch


@pytest.fixture(scope="module")
def l2(cr, torch_):
    return torch_.cuda.get_device_properties(0).L2_cache_size


def assert_same_image(dev, ora, what=""):
    gi = dev.image()
    oi = ora.image()
    for k in ("n_containers", "universe_size", "total_cardinality", "negated", "n_bitmap", "n_array",
              "n_run", "array_pool_bytes", "run_pool_bytes", "max_key"):
        assert gi[k] == oi[k], f"{what}: field {k}: gpu {gi[k]} != oracle {oi[k]}"
    for k in ("keys", "types", "offsets", "cards", "key_index", "bitmap", "array", "run"):
        assert np.array_equal(gi[k], oi[k]), f"{what}: array {k} differs"


def truth_words(ids, universe):
    w = np.zeros(max(1, (universe + 31) // 32), dtype=np.uint32)
    ids = np.unique(np.asarray(ids, dtype=np.uint64))
    if ids.size:
        np.bitwise_or.at(w, (ids // 32).astype(np.int64), (1 << (ids % 32)).astype(np.uint32))
    return w[: (universe + 31) // 32]


def bits_to_bool(words, n):
    return np.unpackbits(np.asarray(words).view(np.uint8), bitorder="little")[:n].astype(bool)


def config1_like(seed=42, n_a=200_000, universe=1 << 22):
    """BASELINE config 1 shapes at reduced size: A uniform IDs with
    duplicates; B alternating gap/run lengths uniform in [1, 4096]."""
    rng = np.random.default_rng(seed)
    a = rng.integers(0, universe, n_a, dtype=np.uint64).astype(np.uint32)
    parts, pos, on = [], 0, False
    while pos < universe:
        ln = int(rng.integers(1, 4097))
        if on:
            parts.append(np.arange(pos, min(pos + ln, universe), dtype=np.uint32))
        pos += ln
        on = not on
    b = np.concatenate(parts)
    return a, b, universe


# --------------------------------------------------------------- uploads

UPLOAD_SETS = ["setops_bb_a", "setops_aa_a", "setops_ba_b", "compl_absent_key", "compl_low",
               "absent_B", "mixed5_1", "alt8_0", "uniform_int_1e6", "setops_disjoint_a"]


@pytest.mark.parametrize("name", UPLOAD_SETS)
@pytest.mark.parametrize("thr", [KEEP, ALL, AUTO, 100])
def test_upload_from_ids_matches_oracle(cr, oracle, l2, name, thr):
    words, u = ref_sets.load(name)
    ids = ref_sets.ids_of(words)
    rng = np.random.default_rng(7)
    shuffled = np.concatenate([ids, ids[: ids.size // 20]])  # ~5% duplicates
    rng.shuffle(shuffled)
    dev = cr.upload_from_ids(shuffled, u, bitmap_threshold=thr)
    ora = oracle.from_ids(shuffled, u, thr, l2)
    assert_same_image(dev, ora, f"{name}/{thr}")
    dev.free()


@pytest.mark.parametrize("name", UPLOAD_SETS[:6])
@pytest.mark.parametrize("thr", [KEEP, ALL, AUTO])
def test_upload_from_bitset_matches_oracle(cr, oracle, l2, torch_, name, thr):
    words, u = ref_sets.load(name)
    ora = oracle.from_bitset(words, u, thr, l2)
    dev = cr.upload_from_bitset(words, u, bitmap_threshold=thr)
    assert_same_image(dev, ora, f"host bitset {name}")
    dev.free()
    dword = torch_.from_numpy(words.view(np.int32)).cuda()
    dev = cr.upload_from_device_bitset(dword, u, bitmap_threshold=thr)
    assert_same_image(dev, ora, f"device bitset {name}")
    dev.free()


def test_upload_device_ids_and_config1(cr, oracle, l2, torch_):
    a, b, u = config1_like()
    for ids in (a, b):
        for thr in (KEEP, ALL, AUTO):
            ora = oracle.from_ids(ids, u, thr, l2)
            dev = cr.upload_from_ids(torch_.from_numpy(ids.view(np.int32)).cuda(), u, bitmap_threshold=thr)
            assert_same_image(dev, ora, f"device ids thr={thr}")
            dev.free()


@pytest.mark.parametrize("case", ["empty", "single", "full_chunk", "tail", "u_not_chunk", "huge_u_sparse"])
def test_upload_edges(cr, oracle, l2, case):
    if case == "empty":
        ids, u = np.zeros(0, np.uint32), 1000
    elif case == "single":
        ids, u = np.array([123456], np.uint32), 1 << 20
    elif case == "full_chunk":
        ids, u = np.arange(65536, 131072, dtype=np.uint32), 10 * 65536
    elif case == "tail":
        ids, u = np.arange(0, 100001, 3, dtype=np.uint32), 100001
    elif case == "u_not_chunk":
        ids, u = np.arange(60000, 70001, dtype=np.uint32), 70001  # > U/2: negated, tail masked
    else:
        ids, u = np.array([0, 4_000_000_000, 17, 2**32 - 2], np.uint32), 2**32 - 1
    for thr in (KEEP, ALL):
        dev = cr.upload_from_ids(ids, u, bitmap_threshold=thr)
        ora = oracle.from_ids(ids, u, thr, l2)
        assert_same_image(dev, ora, case)
        assert np.array_equal(cr.decompress_to_bitset(dev).cpu().numpy().view(np.uint32)
                              if u < 2**31 else np.zeros(0), ora.decompress() if u < 2**31 else np.zeros(0))
        dev.free()


def test_upload_rejects_out_of_universe(cr):
    with pytest.raises(RuntimeError, match="universe"):
        cr.upload_from_ids(np.array([1, 2, 1000], np.uint32), 100)


def mixed_chunks(rng, n_chunks, scale=1.0):
    """Config-2 shapes: sparse (Poisson 2000), dense (Bernoulli 0.3) and run
    chunks (runs of length [256, 8192]) in thirds, ~5% duplicates, shuffled."""
    parts = []
    for c in range(n_chunks):
        base = c << 16
        kind = c % 3
        if kind == 0:
            m = rng.poisson(2000 * scale)
            parts.append(base + rng.integers(0, 65536, m, dtype=np.int64))
        elif kind == 1:
            parts.append(base + np.flatnonzero(rng.random(65536) < 0.3))
        else:
            pos = int(rng.integers(0, 4096))
            while pos < 65536:
                ln = int(rng.integers(256, 8193))
                parts.append(base + np.arange(pos, min(pos + ln, 65536)))
                pos += ln + int(rng.integers(256, 8193))
    ids = np.concatenate(parts).astype(np.uint32)
    ids = np.concatenate([ids, ids[rng.integers(0, ids.size, ids.size // 20)]])
    rng.shuffle(ids)
    return ids


@pytest.mark.parametrize("case", ["u26", "u26_unaligned", "u31_many_passes", "u26_uniform"])
def test_upload_large_dense(cr, oracle, l2, torch_, case):
    """Large dense uploads (>= 2^22 IDs: several scatter passes over chunk
    slot ranges, more than 32768 chunks, a ragged tail, an unaligned ID
    pointer) give the oracle's image."""
    rng = np.random.default_rng(11)
    if case == "u31_many_passes":
        u = (1 << 31) + 12345  # 32769 chunks: eight scatter passes
        ids = rng.integers(0, u, 40_000_037, dtype=np.uint64).astype(np.uint32)
        thrs = (AUTO,)
    elif case == "u26_uniform":
        u = 1 << 26
        ids = rng.integers(0, u, (1 << 22) + 5, dtype=np.uint64).astype(np.uint32)
        thrs = (KEEP, ALL)
    else:
        u = 1 << 26
        ids = mixed_chunks(rng, 1024)
        thrs = (KEEP, ALL, AUTO)
    assert ids.size >= 1 << 22
    d = torch_.from_numpy(np.concatenate([np.zeros(1, np.uint32), ids]).view(np.int32)).cuda()
    src = d[1:] if case == "u26_unaligned" else d[1:].clone()
    for thr in thrs:
        ora = oracle.from_ids(ids, u, thr, l2)
        dev = cr.upload_from_ids(src, u, bitmap_threshold=thr)
        assert_same_image(dev, ora, f"{case} thr={thr}")
        dev.free()


def test_upload_large_rejects_out_of_universe(cr, torch_):
    ids = np.arange(0, 1 << 23, dtype=np.uint32)
    ids[5_000_001] = 1 << 23
    with pytest.raises(RuntimeError, match="universe"):
        cr.upload_from_ids(torch_.from_numpy(ids.view(np.int32)).cuda(), 1 << 23)


# ------------------------------------------------------------ set algebra

def forced_negated(cr, oracle, words, u):
    """Stored = complement of `words`, negated=true (the reference's
    DeMorgan test operands, test/test_complement.cu:372-397)."""
    comp = ~words
    if u % 32:
        comp[-1] &= (1 << (u % 32)) - 1
    card = int(bits_to_bool(words, u).sum())
    d = cr.upload_from_bitset(comp, u * 4, bitmap_threshold=KEEP)
    d.raw.negated = 1
    d.raw.universe_size = u
    d.raw.total_cardinality = card
    o = oracle.from_bitset(comp, u * 4, KEEP)
    o.im.negated = 1
    o.im.universe_size = u
    o.im.total_cardinality = card
    return d, o


@pytest.mark.parametrize("op", [AND, OR, ANDNOT, XOR])
@pytest.mark.parametrize("na,nb", [(False, False), (True, False), (False, True), (True, True)])
def test_demorgan_16(cr, oracle, op, na, nb):
    wa, u = ref_sets.load("demorgan_a")
    wb, _ = ref_sets.load("demorgan_b")
    da, oa = forced_negated(cr, oracle, wa, u) if na else (cr.upload_from_bitset(wa, u, bitmap_threshold=KEEP),
                                                          oracle.from_bitset(wa, u, KEEP))
    db, ob = forced_negated(cr, oracle, wb, u) if nb else (cr.upload_from_bitset(wb, u, bitmap_threshold=KEEP),
                                                          oracle.from_bitset(wb, u, KEEP))
    dr = cr.set_operation(da, db, op)
    orr = oracle.set_operation(oa, ob, op)
    assert_same_image(dr, orr, f"demorgan op={op} na={na} nb={nb}")
    want = {AND: wa & wb, OR: wa | wb, ANDNOT: wa & ~wb, XOR: wa ^ wb}[op]
    got = cr.decompress_to_bitset(dr).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, want)
    for x in (dr, da, db):
        x.free()


SETOPS = [("setops_bb_a", "setops_bb_b"), ("setops_aa_a", "setops_aa_b"), ("setops_ba_a", "setops_ba_b"),
          ("setops_disjoint_a", "setops_disjoint_b"), ("setops_ident", "setops_ident"),
          ("setops_xor_ident", "setops_xor_ident"), ("setops_aa_a", "setops_bb_b")]


@pytest.mark.parametrize("an,bn", SETOPS)
@pytest.mark.parametrize("op", [AND, OR, ANDNOT, XOR])
@pytest.mark.parametrize("ta,tb", [(KEEP, KEEP), (ALL, ALL), (KEEP, ALL)])
def test_setops_match_oracle(cr, oracle, an, bn, op, ta, tb):
    wa, u = ref_sets.load(an)
    wb, _ = ref_sets.load(bn)
    ua = 2 * u  # a larger universe: no automatic complement
    da, db = cr.upload_from_bitset(wa, ua, bitmap_threshold=ta), cr.upload_from_bitset(wb, ua, bitmap_threshold=tb)
    oa, ob = oracle.from_bitset(wa, ua, ta), oracle.from_bitset(wb, ua, tb)
    dr = cr.set_operation(da, db, op)
    assert_same_image(dr, oracle.set_operation(oa, ob, op), f"{an},{bn},op={op}")
    for x in (dr, da, db):
        x.free()


def test_setops_with_runs(cr, oracle, l2):
    a, b, u = config1_like(seed=3, n_a=50_000, universe=1 << 21)
    da, db = cr.upload_from_ids(a, u, bitmap_threshold=KEEP), cr.upload_from_ids(b, u, bitmap_threshold=KEEP)
    oa, ob = oracle.from_ids(a, u, KEEP, l2), oracle.from_ids(b, u, KEEP, l2)
    assert db.raw.n_run_containers > 0
    for op in (AND, OR, ANDNOT, XOR):
        dr = cr.set_operation(da, db, op)
        assert_same_image(dr, oracle.set_operation(oa, ob, op), f"runs op={op}")
        dr = cr.set_operation(db, da, op)
        assert_same_image(dr, oracle.set_operation(ob, oa, op), f"runs swapped op={op}")
        dr.free()


MULTI = [(["setops_mand_a", "setops_mand_b", "setops_mand_c"], "and"),
         (["setops_mor_a", "setops_mor_b", "setops_mor_c"], "or"),
         (["mand_neg_1", "mand_neg_2", "mand_neg_3"], "and"),
         (["mand_allneg_1", "mand_allneg_2", "mand_allneg_3"], "and"),
         (["mand_allneg_1", "mand_allneg_2", "mand_allneg_3"], "or"),
         (["absent_A", "absent_B", "absent_C"], "and"),
         ([f"mixed5_{i}" for i in range(5)], "and"),
         ([f"alt8_{i}" for i in range(8)], "and"),
         ([f"alt8_{i}" for i in range(8)], "or"),
         (["setops_mand_a"], "and")]


@pytest.mark.parametrize("names,fn", MULTI)
@pytest.mark.parametrize("thr", [ALL, KEEP])
def test_multi_matches_oracle(cr, oracle, l2, names, fn, thr):
    sets = [ref_sets.load(n) for n in names]
    dev = [cr.upload_from_bitset(w, u, bitmap_threshold=thr) for w, u in sets]
    ora = [oracle.from_bitset(w, u, thr, l2) for w, u in sets]
    dr = (cr.multi_and if fn == "and" else cr.multi_or)(dev)
    orr = (oracle.multi_and if fn == "and" else oracle.multi_or)(ora)
    assert_same_image(dr, orr, f"multi_{fn} {names[0]}")
    want = sets[0][0].copy()
    for w, _ in sets[1:]:
        want = (want & w) if fn == "and" else (want | w)
    assert np.array_equal(cr.decompress_to_bitset(dr).cpu().numpy().view(np.uint32), want)
    for x in dev + [dr]:
        x.free()


# --------------------------------------------------- queries and export

@pytest.mark.parametrize("name", ["setops_bb_a", "setops_aa_b", "compl_absent_key", "absent_B", "alt8_1"])
@pytest.mark.parametrize("thr", [KEEP, ALL])
def test_contains_matches_oracle(cr, oracle, torch_, name, thr):
    words, u = ref_sets.load(name)
    dev = cr.upload_from_bitset(words, u, bitmap_threshold=thr)
    ora = oracle.from_bitset(words, u, thr)
    rng = np.random.default_rng(11)
    uniform = rng.integers(0, u + 70000, 300_001, dtype=np.uint64).astype(np.uint32)
    starts = rng.integers(0, u, 5000, dtype=np.uint64).astype(np.uint32)
    blocks = (starts[:, None] + np.arange(32, dtype=np.uint32)[None, :]).reshape(-1)
    for q in (uniform, blocks):
        want = ora.contains(q)
        dq = torch_.from_numpy(q.view(np.int32)).cuda()
        for warp in (False, True):
            got = cr.contains_batch(dev, dq, warp=warp).cpu().numpy().view(np.uint32)
            assert np.array_equal(got, want), f"{name} warp={warp}"
    dev.free()


@pytest.mark.parametrize("name", ["setops_bb_a", "setops_aa_b", "compl_absent_key", "absent_B",
                                  "uniform_int_1e6"])
@pytest.mark.parametrize("thr", [KEEP, ALL])
def test_decompress_enumerate_promote(cr, oracle, torch_, name, thr):
    words, u = ref_sets.load(name)
    dev = cr.upload_from_bitset(words, u, bitmap_threshold=thr)
    ora = oracle.from_bitset(words, u, thr)
    got = cr.decompress_to_bitset(dev).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, words)
    big = torch_.full(((u + 31) // 32 + 5000,), -1, dtype=torch_.int32, device="cuda")
    got = cr.decompress_to_bitset(dev, output=big).cpu().numpy().view(np.uint32)
    assert np.array_equal(got[: words.size], words) and not got[words.size:].any()
    ids = ref_sets.ids_of(words)
    assert np.array_equal(cr.enumerate_ids(dev).cpu().numpy(), ids.astype(np.int64))
    assert np.array_equal(cr.enumerate_ids(dev, dtype="uint32").cpu().numpy().view(np.uint32), ids)
    p = cr.promote_to_bitmap(dev)
    assert_same_image(p, oracle.promote_to_bitmap(ora), "promote")
    c = cr.gpu_roaring_deep_copy(dev)
    assert_same_image(c, ora, "deep copy")
    for x in (dev, p, c):
        x.free()


def test_promote_auto_and_resolve(cr, oracle, l2):
    assert cr.resolve_auto_threshold(1_000_000) == KEEP
    assert cr.resolve_auto_threshold(1_000_000_000) == ALL
    words, u = ref_sets.load("setops_aa_a")
    dev = cr.upload_from_bitset(words, u, bitmap_threshold=KEEP)
    small = cr.promote_auto(dev)
    assert small.raw.n_array_containers == dev.raw.n_array_containers  # fits L2: deep copy
    ids = ref_sets.ids_of(words)
    big_u = 1_000_000_000
    dev2 = cr.upload_from_ids(ids, big_u, bitmap_threshold=KEEP)
    promoted = cr.promote_auto(dev2)
    assert promoted.raw.n_array_containers == 0 and promoted.raw.n_bitmap_containers == dev2.raw.n_containers
    for x in (dev, small, dev2, promoted):
        x.free()


def test_cpp_dropin_program(built_lib, cr):
    """The C++ user program over the public headers (tests/cpp/api_test.cu)."""
    import subprocess

    import build

    exe = build.build_cpp_tests()
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "0 failed" in res.stdout


@pytest.mark.parametrize("count", [65, 130])
@pytest.mark.parametrize("fn", ["and", "or"])
def test_multi_more_than_64_inputs(cr, oracle, l2, count, fn):
    """More inputs than one k-way pass takes (the reference accepts any
    count, src/set_ops.cu:1733-1762): chained passes of 64, bit-exact against
    the oracle's identical chaining and against numpy. Dense inputs (most
    stored as complements) keep the AND non-empty; every 7th input is sparse."""
    u = 1 << 18
    rng = np.random.default_rng(count)
    sets = []
    for i in range(count):
        p = 0.02 if i % 7 == 3 else 0.995
        ids = np.flatnonzero(rng.random(u) < p).astype(np.uint32)
        sets.append(truth_words(ids, u))
    dev = [cr.upload_from_bitset(w, u) for w in sets]
    ora = [oracle.from_bitset(w, u, AUTO, l2) for w in sets]
    assert any(d.raw.negated for d in dev) and not all(d.raw.negated for d in dev)
    dr = (cr.multi_and if fn == "and" else cr.multi_or)(dev)
    orr = (oracle.multi_and if fn == "and" else oracle.multi_or)(ora)
    assert_same_image(dr, orr, f"multi_{fn} x{count}")
    want = sets[0].copy()
    for w in sets[1:]:
        want = (want & w) if fn == "and" else (want | w)
    assert np.array_equal(cr.decompress_to_bitset(dr).cpu().numpy().view(np.uint32), want)
    for x in dev + [dr]:
        x.free()
