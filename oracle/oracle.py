"""ctypes binding of the CPU oracle (oracle/roaring_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm, never by the product path.
Images are returned as dicts with the same keys as
cu_roaring_b200.GpuRoaring.image() so results compare field by field.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"


def build() -> Path:
    src = [HERE / "roaring_oracle.c", HERE / "roaring_oracle.h", HERE / "cpu_upload.cpp", HERE / "Makefile"]
    if not LIB.exists() or LIB.stat().st_mtime < max(p.stat().st_mtime for p in src):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


class Image(C.Structure):
    _fields_ = [
        ("n_containers", C.c_uint32), ("universe_size", C.c_uint32),
        ("total_cardinality", C.c_uint64), ("n_bitmap", C.c_uint32), ("n_array", C.c_uint32),
        ("n_run", C.c_uint32), ("array_pool_bytes", C.c_uint32), ("run_pool_bytes", C.c_uint32),
        ("max_key", C.c_uint32), ("negated", C.c_int32),
        ("keys", C.POINTER(C.c_uint16)), ("types", C.POINTER(C.c_uint8)),
        ("offsets", C.POINTER(C.c_uint32)), ("cards", C.POINTER(C.c_uint16)),
        ("key_index", C.POINTER(C.c_uint16)), ("bitmap", C.POINTER(C.c_uint64)),
        ("array", C.POINTER(C.c_uint16)), ("run", C.POINTER(C.c_uint16)),
    ]


_lib = None
_IP = C.POINTER(Image)


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB))
        v, u32, u64, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int
        sig = {
            "or_image_free": ([_IP], None),
            "or_container_type": ([u32, u32, u32], i32),
            "or_resolve_auto_threshold": ([u32, u64], u32),
            "or_from_ids": ([v, u64, u32, u32, u64, _IP], i32),
            "or_from_bitset": ([v, u64, u32, u32, u64, _IP], i32),
            "or_set_operation": ([_IP, _IP, i32, _IP], i32),
            "or_multi_and": ([C.POINTER(_IP), u32, _IP], i32),
            "or_multi_or": ([C.POINTER(_IP), u32, _IP], i32),
            "or_promote_to_bitmap": ([_IP, _IP], i32),
            "or_contains_batch": ([_IP, v, u64, v, i32], None),
            "or_decompress": ([_IP, v, u64], None),
            "or_enumerate": ([_IP, v], u64),
            "or_validate": ([_IP], i32),
            "or_topk": ([v, u64, u32, v, u32, v, u32, i32, v, v, i32], None),
            "or_topk_f32": ([v, v, u64, u32, v, u32, v, u32, i32, v, v, i32], None),
            "or_widen_f16": ([v, u64, v], None),
            "or_row_norms_f32": ([v, u64, u32, v], None),
            "or_cpu_upload_sorted": ([v, u64, u32, u32, v], u64),
            "or_serialize_portable": ([v, u64, i32, v, u64], u64),
        }
        for name, (a, r) in sig.items():
            f = getattr(_lib, name)
            f.argtypes = a
            f.restype = r
    return _lib


# B200: 126 MiB of L2 as cudaDevAttrL2CacheSize reports it. Tests pass the
# device's own value where it matters.
B200_L2 = 132_120_576


class OracleBitmap:
    """Owns one oracle image."""

    def __init__(self):
        self.im = Image()

    def __del__(self):
        if _lib is not None and getattr(self, "im", None) is not None:
            _lib.or_image_free(C.byref(self.im))

    def image(self) -> dict:
        im = self.im
        n = im.n_containers

        def arr(ptr, count, dtype):
            if count == 0 or not ptr:
                return np.zeros(0, dtype=dtype)
            return np.ctypeslib.as_array(ptr, shape=(count,)).astype(dtype, copy=True)

        return {
            "n_containers": n, "universe_size": im.universe_size,
            "total_cardinality": im.total_cardinality, "negated": bool(im.negated),
            "n_bitmap": im.n_bitmap, "n_array": im.n_array, "n_run": im.n_run,
            "array_pool_bytes": im.array_pool_bytes, "run_pool_bytes": im.run_pool_bytes,
            "max_key": im.max_key if n else 0,
            "keys": arr(im.keys, n, np.uint16), "types": arr(im.types, n, np.uint8),
            "offsets": arr(im.offsets, n, np.uint32), "cards": arr(im.cards, n, np.uint16),
            "key_index": arr(im.key_index, (im.max_key + 1) if n else 0, np.uint16),
            "bitmap": arr(im.bitmap, im.n_bitmap * 1024, np.uint64),
            "array": arr(im.array, im.array_pool_bytes // 2, np.uint16),
            "run": arr(im.run, im.run_pool_bytes // 2, np.uint16),
        }

    def validate(self) -> int:
        return lib().or_validate(C.byref(self.im))

    def contains(self, ids: np.ndarray, threads: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((ids.size + 31) // 32, dtype=np.uint32)
        lib().or_contains_batch(C.byref(self.im), ids.ctypes.data, ids.size, out.ctypes.data,
                                threads or os.cpu_count() or 1)
        return out

    def decompress(self, n_words: int | None = None) -> np.ndarray:
        if n_words is None:
            n_words = (self.im.universe_size + 31) // 32
        out = np.zeros(max(1, n_words), dtype=np.uint32)
        lib().or_decompress(C.byref(self.im), out.ctypes.data, n_words)
        return out[:n_words]

    def enumerate(self) -> np.ndarray:
        n = lib().or_enumerate(C.byref(self.im), None)
        out = np.zeros(max(1, n), dtype=np.uint32)
        lib().or_enumerate(C.byref(self.im), out.ctypes.data)
        return out[:n]


def container_type(c: int, r: int, t: int) -> int:
    return lib().or_container_type(c, r, t)


def resolve_auto_threshold(universe: int, l2_bytes: int = B200_L2) -> int:
    return lib().or_resolve_auto_threshold(universe, l2_bytes)


def from_ids(ids, universe: int, threshold: int = 0xFFFFFFFF, l2_bytes: int = B200_L2) -> OracleBitmap:
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    b = OracleBitmap()
    rc = lib().or_from_ids(ids.ctypes.data if ids.size else None, ids.size, universe, threshold,
                           l2_bytes, C.byref(b.im))
    if rc != 0:
        raise ValueError(f"or_from_ids: {rc}")
    return b


def from_bitset(words, universe: int, threshold: int = 0xFFFFFFFF, l2_bytes: int = B200_L2) -> OracleBitmap:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    b = OracleBitmap()
    lib().or_from_bitset(words.ctypes.data if words.size else None, words.size, universe, threshold,
                         l2_bytes, C.byref(b.im))
    return b


def cpu_upload_sorted(ids, universe: int, threshold: int) -> dict:
    """The reference's host upload path restated (sort, unique, complement,
    partition, pools); CPU baseline timing only. Returns its counts."""
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    cnt = np.zeros(4, dtype=np.uint64)
    lib().or_cpu_upload_sorted(ids.ctypes.data if ids.size else None, ids.size, universe, threshold,
                               cnt.ctypes.data)
    return {"containers": int(cnt[0]), "bitmaps": int(cnt[1]), "arrays": int(cnt[2]), "cardinality": int(cnt[3])}


def set_operation(a: OracleBitmap, b: OracleBitmap, op: int) -> OracleBitmap:
    r = OracleBitmap()
    lib().or_set_operation(C.byref(a.im), C.byref(b.im), op, C.byref(r.im))
    return r


def _multi(fn, bms) -> OracleBitmap:
    r = OracleBitmap()
    arr = (_IP * max(1, len(bms)))(*[C.pointer(b.im) for b in bms])
    fn(arr, len(bms), C.byref(r.im))
    return r


def multi_and(bms) -> OracleBitmap:
    return _multi(lib().or_multi_and, bms)


def multi_or(bms) -> OracleBitmap:
    return _multi(lib().or_multi_or, bms)


def promote_to_bitmap(a: OracleBitmap) -> OracleBitmap:
    r = OracleBitmap()
    lib().or_promote_to_bitmap(C.byref(a.im), C.byref(r.im))
    return r


def serialize_portable(ids, allow_runs: bool = True) -> bytes:
    """Portable Roaring serialization of a set of uint32 IDs (any order, duplicates ok)."""
    a = np.unique(np.asarray(ids, dtype=np.uint32))
    f = lib().or_serialize_portable
    n = f(a.ctypes.data if a.size else None, C.c_uint64(a.size), int(allow_runs), None, C.c_uint64(0))
    buf = (C.c_uint8 * max(1, n))()
    f(a.ctypes.data if a.size else None, C.c_uint64(a.size), int(allow_runs), buf, C.c_uint64(n))
    return bytes(buf)[:n]


def topk(db_f16: np.ndarray, queries_f16: np.ndarray, k: int, metric: int = 0,
         pass_bits: np.ndarray | None = None, threads: int = 0):
    db = np.ascontiguousarray(db_f16).view(np.uint16)
    q = np.ascontiguousarray(queries_f16).view(np.uint16)
    n, d = db.shape
    nq = q.shape[0]
    dist = np.zeros((nq, k), dtype=np.float32)
    ids = np.zeros((nq, k), dtype=np.int64)
    pb = None if pass_bits is None else np.ascontiguousarray(pass_bits, dtype=np.uint32)
    lib().or_topk(db.ctypes.data, n, d, q.ctypes.data, nq, pb.ctypes.data if pb is not None else None,
                  k, metric, dist.ctypes.data, ids.ctypes.data, threads or os.cpu_count() or 1)
    return dist, ids


class F32Database:
    """A database widened to fp32 once, for repeated timed CPU top-k calls."""

    def __init__(self, db_f16: np.ndarray):
        h = np.ascontiguousarray(db_f16).view(np.uint16)
        self.n, self.dim = h.shape
        self.f = np.empty((self.n, self.dim), dtype=np.float32)
        lib().or_widen_f16(h.ctypes.data, h.size, self.f.ctypes.data)
        self.norms = np.empty(self.n, dtype=np.float32)
        lib().or_row_norms_f32(self.f.ctypes.data, self.n, self.dim, self.norms.ctypes.data)

    def topk(self, queries_f16, k, metric=0, pass_bits=None, threads=0):
        q = np.ascontiguousarray(queries_f16).view(np.uint16)
        nq = q.shape[0]
        dist = np.zeros((nq, k), dtype=np.float32)
        ids = np.zeros((nq, k), dtype=np.int64)
        pb = None if pass_bits is None else np.ascontiguousarray(pass_bits, dtype=np.uint32)
        lib().or_topk_f32(self.f.ctypes.data, self.norms.ctypes.data, self.n, self.dim, q.ctypes.data, nq,
                          pb.ctypes.data if pb is not None else None, k, metric, dist.ctypes.data,
                          ids.ctypes.data, threads or os.cpu_count() or 1)
        return dist, ids
