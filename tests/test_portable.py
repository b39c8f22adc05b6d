"""Portable Roaring serialization: the oracle's writer against known answers
derived by hand from the published format specification (CPU), the
ingest's header validation through the C ABI (CPU, before any device work),
and cr_upload_portable against the bitset upload of the same set (GPU)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import ref_sets


def test_oracle_writer_known_answers(oracle):
    # No run containers: cookie 12346, 2 containers, (key, card-1) headers,
    # offsets 24 and 30, then the two ARRAY payloads.
    want = bytes.fromhex("3a300000" "02000000" "00000200" "01000000" "18000000" "1e000000"
                         "010002000300" "0500")
    assert oracle.serialize_portable([3, 1, 2, 65541, 2], allow_runs=False) == want
    # One RUN container: cookie 12347 | (1 - 1) << 16, run-flag byte, header
    # (key 0, card-1 99), no offsets below 4 containers, run count 1, (100, 99).
    want = bytes.fromhex("3b300000" "01" "00006300" "0100" "6400" "6300")
    assert oracle.serialize_portable(range(100, 200)) == want
    # A BITMAP container: 8192 payload bytes, bit i at byte i/8.
    ids = np.arange(0, 65536, 3, dtype=np.uint32)
    b = oracle.serialize_portable(ids, allow_runs=False)
    assert len(b) == 8 + 4 + 4 + 8192 and b[16] == 0b01001001


def _call(cr, data: bytes, universe: int):
    out = cr.GpuRoaring()
    buf = C.create_string_buffer(data, len(data))
    rc = cr.lib().cr_upload_portable(C.cast(buf, C.c_void_p), len(data), universe, None, cr.PROMOTE_AUTO,
                                     C.byref(out.raw))
    return rc, cr.lib().cr_last_error_string()


def test_ingest_rejects_malformed_headers(built_lib, oracle):
    import cu_roaring_b200 as cr

    good = oracle.serialize_portable([1, 2, 3, 65541], allow_runs=False)
    rc, msg = _call(cr, b"\x00\x01\x02\x03" + good[4:], 1 << 20)
    assert rc == -1 and b"cookie" in msg
    rc, msg = _call(cr, good[:20], 1 << 20)
    assert rc == -1 and b"truncated" in msg
    rc, msg = _call(cr, good, 65536)  # the second container is key 1: past a 65536-ID universe
    assert rc == -4 and b"universe" in msg
    swapped = bytearray(good)
    swapped[8:12], swapped[12:16] = good[12:16], good[8:12]  # keys out of order
    rc, msg = _call(cr, bytes(swapped), 1 << 20)
    assert rc == -1 and b"increasing" in msg


def _sets():
    rng = np.random.default_rng(5)
    U = 1 << 22
    mixed = []
    for chunk in range(U >> 16):
        base = chunk << 16
        if chunk % 3 == 0:
            mixed.append(base + rng.choice(65536, 700, replace=False))
        elif chunk % 3 == 1:
            mixed.append(base + np.flatnonzero(rng.random(65536) < 0.4))
        else:
            starts = np.sort(rng.choice(65536 - 3000, 12, replace=False))
            mixed.append(np.concatenate([base + np.arange(s, s + int(rng.integers(1, 3000))) for s in starts]))
    out = [("mixed", np.unique(np.concatenate(mixed)).astype(np.uint32), U),
           ("dense_complement", np.flatnonzero(rng.random(U) < 0.8).astype(np.uint32), U),
           ("tail_universe", np.array([0, 5, 70000, 70001, 99999], dtype=np.uint32), 100000),
           ("empty", np.array([], dtype=np.uint32), 1 << 20)]
    for name in ("setops_bb_a", "compl_absent_key", "uniform_int_1e6"):
        words, u = ref_sets.load(name)
        out.append((name, ref_sets.ids_of(words).astype(np.uint32), u))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("allow_runs", [True, False])
@pytest.mark.parametrize("thr", [4096, 0])
def test_ingest_matches_bitset_upload(cr, oracle, allow_runs, thr):
    from test_gpu_parity import assert_same_image

    for name, ids, U in _sets():
        data = oracle.serialize_portable(ids, allow_runs=allow_runs)
        words = np.zeros(max(1, (U + 31) // 32), dtype=np.uint32)
        np.bitwise_or.at(words, ids // 32, (np.uint32(1) << (ids % 32)).astype(np.uint32))
        want = cr.upload_from_bitset(words, U, bitmap_threshold=thr)
        got = cr.upload_portable(data, U, bitmap_threshold=thr)
        assert_same_image(got, want, f"{name} runs={allow_runs} thr={thr}")
        got.free()
        want.free()


@pytest.mark.gpu
def test_ingest_rejects_device_side_errors(cr, oracle):
    """Checks that need the payload: a member past a universe that ends inside
    the last container, and a declared cardinality the payload does not have."""
    data = oracle.serialize_portable([1, 2, 99990, 99999], allow_runs=False)
    rc, msg = _call(cr, data, 99995)
    assert rc == -4 and b"universe" in msg
    bad = bytearray(data)
    bad[10] = 5  # container 0 declares 6 members, its payload holds 4 (plus the next header bytes)
    rc, msg = _call(cr, bytes(bad), 1 << 20)
    assert rc == -1


def _decode_portable(b: bytes) -> np.ndarray:
    """A pure-Python reader of the portable Roaring format, written from the
    published specification (independent of the C writer under test)."""
    import struct

    cookie = struct.unpack_from("<I", b, 0)[0]
    if cookie & 0xFFFF == 12347:
        n = (cookie >> 16) + 1
        runs = b[4:4 + (n + 7) // 8]
        pos = 4 + (n + 7) // 8
        is_run = [(runs[i // 8] >> (i % 8)) & 1 for i in range(n)]
        has_off = n >= 4
    else:
        assert cookie == 12346
        n = struct.unpack_from("<I", b, 4)[0]
        pos = 8
        is_run = [0] * n
        has_off = True
    hdr = [struct.unpack_from("<HH", b, pos + 4 * i) for i in range(n)]
    pos += 4 * n
    offs = [struct.unpack_from("<I", b, pos + 4 * i)[0] for i in range(n)] if has_off else None
    if has_off:
        pos += 4 * n
    out = []
    for i, (key, card_m1) in enumerate(hdr):
        card = card_m1 + 1
        at = offs[i] if offs else pos
        if is_run[i]:
            nr = struct.unpack_from("<H", b, at)[0]
            pairs = np.frombuffer(b, dtype="<u2", count=2 * nr, offset=at + 2).reshape(nr, 2).astype(np.int64)
            vals = np.concatenate([np.arange(s, s + l + 1) for s, l in pairs]) if nr else np.zeros(0, np.int64)
            size = 2 + 4 * nr
        elif card <= 4096:
            vals = np.frombuffer(b, dtype="<u2", count=card, offset=at).astype(np.int64)
            size = 2 * card
        else:
            words = np.frombuffer(b, dtype="<u8", count=1024, offset=at)
            bits = np.unpackbits(words.view(np.uint8), bitorder="little")
            vals = np.flatnonzero(bits).astype(np.int64)
            size = 8192
        assert vals.size == card, f"container {i}: {vals.size} members, header says {card}"
        out.append((key << 16) + vals)
        pos = at + size
    return np.concatenate(out).astype(np.uint32) if out else np.zeros(0, np.uint32)


@pytest.mark.parametrize("allow_runs", [True, False])
def test_oracle_writer_round_trips_through_spec_reader(oracle, allow_runs):
    rng = np.random.default_rng(17)
    parts = []
    for chunk in range(12):
        base = chunk << 16
        kind = chunk % 4
        if kind == 0:
            parts.append(base + rng.choice(65536, 300, replace=False))
        elif kind == 1:
            parts.append(base + np.flatnonzero(rng.random(65536) < 0.5))
        elif kind == 2:
            parts.append(base + np.arange(1000, 40000))
        # kind 3: absent chunk
    ids = np.unique(np.concatenate(parts)).astype(np.uint32)
    for subset in (ids, ids[:5], ids[ids < (3 << 16)]):
        got = _decode_portable(oracle.serialize_portable(subset, allow_runs=allow_runs))
        assert np.array_equal(got, subset)
