"""Python host mirror of the cu_roaring C++ API over libcuroaring_b200.so.

The names, argument meanings and error behaviour follow the reference's C++
API (include/cu_roaring/detail/*.cuh): functions return GpuRoaring owners,
failures raise RuntimeError (the reference throws std::runtime_error from
CUDA_CHECK, include/cu_roaring/detail/utils.cuh:9-18). Device buffers are
torch CUDA tensors (plumbing only); every computation is a call through the
C ABI into the sm_100a kernels. There is no CPU fallback: importing this
module without the built library raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libcuroaring_b200.so"
if not _LIB_PATH.exists():
    raise ImportError(f"{_LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
_lib = C.CDLL(str(_LIB_PATH))

PROMOTE_KEEP_DEFAULT = 4096
PROMOTE_ALL = 0
PROMOTE_AUTO = 0xFFFFFFFF

AND, OR, ANDNOT, XOR = 0, 1, 2, 3
ARRAY, BITMAP, RUN = 0, 1, 2
METRIC_IP, METRIC_L2 = 0, 1

EXPORTED_SYMBOLS = (
    "cr_last_error_string", "cr_version", "cr_upload_from_ids", "cr_upload_from_device_ids",
    "cr_upload_from_bitset", "cr_upload_from_device_bitset", "cr_gpu_roaring_free",
    "cr_gpu_roaring_free_async", "cr_resolve_auto_threshold", "cr_promote_to_bitmap",
    "cr_promote_auto", "cr_deep_copy", "cr_set_operation", "cr_multi_and", "cr_multi_or",
    "cr_decompress_to_bitset", "cr_decompress_to_bitset_alloc", "cr_enumerate_ids_i64",
    "cr_enumerate_ids_u32", "cr_enumerate_ids_alloc", "cr_enumerate_ids_u32_noalloc", "cr_contains_batch", "cr_filtered_topk",
    "cr_row_norms", "cr_topk_merge", "cr_topk_merge_packed", "cr_upload_portable", "cr_batch_upload_portable", "cr_batch_free",
    "cr_batch_promote", "cr_batch_multi_and", "cr_batch_decompress", "cr_batch_contains", "cr_filtered_topk_check", "cr_profile_enable", "cr_profile_kinds", "cr_profile_last_ms", "cr_profile_sum_ms",
    "cr_topk_comm_unique_id", "cr_topk_comm_init", "cr_topk_comm_size", "cr_topk_comm_destroy",
    "cr_filtered_topk_sharded", "cr_upload_portable_ex", "cr_portable_meta", "cr_key_range", "cr_key_slice",
    "cr_concat_key_slices", "cr_test_fail_allocations",
)


class CrGpuRoaring(C.Structure):
    """Byte layout of cu_roaring::GpuRoaring (reference include/cu_roaring/types.cuh:15-54)."""

    _fields_ = [
        ("keys", C.c_void_p), ("types", C.c_void_p), ("offsets", C.c_void_p),
        ("cardinalities", C.c_void_p), ("n_containers", C.c_uint32),
        ("universe_size", C.c_uint32), ("total_cardinality", C.c_uint64),
        ("bitmap_data", C.c_void_p), ("n_bitmap_containers", C.c_uint32),
        ("array_data", C.c_void_p), ("n_array_containers", C.c_uint32),
        ("array_pool_bytes", C.c_uint32), ("run_data", C.c_void_p),
        ("n_run_containers", C.c_uint32), ("run_pool_bytes", C.c_uint32),
        ("key_index", C.c_void_p), ("max_key", C.c_uint32), ("negated", C.c_uint8),
        ("_alloc_base", C.c_void_p),
    ]


_P = C.POINTER(CrGpuRoaring)
_vp, _u32, _u64, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int
_sigs = {
    "cr_last_error_string": ([], C.c_char_p),
    "cr_version": ([], C.c_char_p),
    "cr_upload_from_ids": ([_vp, _u32, _u32, _vp, _u32, _P], _i32),
    "cr_upload_from_device_ids": ([_vp, _u64, _u32, _vp, _u32, _P], _i32),
    "cr_upload_from_bitset": ([_vp, _u32, _u32, _vp, _u32, _P], _i32),
    "cr_upload_from_device_bitset": ([_vp, _u32, _u32, _vp, _u32, _P], _i32),
    "cr_gpu_roaring_free": ([_P], _i32),
    "cr_gpu_roaring_free_async": ([_P, _vp], _i32),
    "cr_resolve_auto_threshold": ([_u32, _i32, C.POINTER(_u32)], _i32),
    "cr_promote_to_bitmap": ([_P, _vp, _P], _i32),
    "cr_promote_auto": ([_P, _vp, _i32, _P], _i32),
    "cr_deep_copy": ([_P, _vp, _P], _i32),
    "cr_set_operation": ([_P, _P, _i32, _vp, _P], _i32),
    "cr_multi_and": ([_P, _u32, _vp, _P], _i32),
    "cr_multi_or": ([_P, _u32, _vp, _P], _i32),
    "cr_decompress_to_bitset": ([_P, _vp, _u32, _vp], _i32),
    "cr_decompress_to_bitset_alloc": ([_P, _vp, C.POINTER(_vp)], _i32),
    "cr_enumerate_ids_i64": ([_P, _vp, _vp], _i32),
    "cr_enumerate_ids_u32": ([_P, _vp, _vp], _i32),
    "cr_enumerate_ids_alloc": ([_P, _vp, C.POINTER(_vp)], _i32),
    "cr_enumerate_ids_u32_noalloc": ([_P, _vp, _vp], _i32),
    "cr_contains_batch": ([_P, _vp, _u64, _vp, _i32, _vp], _i32),
    "cr_filtered_topk": ([_vp, _vp, _u64, _u32, _vp, _u32, _P, _u64, _u32, _i32, _vp, _vp, _vp], _i32),
    "cr_row_norms": ([_vp, _u64, _u32, _vp, _vp], _i32),
    "cr_topk_merge": ([_vp, _vp, _u32, _u32, _u32, _i32, _vp, _vp, _vp], _i32),
    "cr_profile_enable": ([_i32], _i32),
    "cr_profile_kinds": ([C.c_uint32], _i32),
    "cr_profile_last_ms": ([_i32, C.POINTER(C.c_float)], _i32),
    "cr_topk_merge_packed": ([C.c_void_p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, _i32, C.c_void_p,
                              C.c_void_p, C.c_void_p], _i32),
    "cr_upload_portable": ([C.c_void_p, C.c_uint64, C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p], _i32),
    "cr_batch_upload_portable": ([C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p], _i32),
    "cr_batch_free": ([C.c_void_p], _i32),
    "cr_batch_promote": ([C.c_void_p, C.c_void_p, C.c_void_p], _i32),
    "cr_batch_multi_and": ([C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p], _i32),
    "cr_batch_decompress": ([C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p], _i32),
    "cr_batch_contains": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p], _i32),
    "cr_filtered_topk_check": ([], _i32),
    "cr_profile_sum_ms": ([_i32, C.POINTER(C.c_float), C.POINTER(C.c_uint32)], _i32),
    "cr_test_fail_allocations": ([C.c_int64], _i32),
    "cr_key_range": ([_u32, _u32, _u32, C.POINTER(_u32), C.POINTER(_u32)], _i32),
    "cr_key_slice": ([_P, _u32, _u32, _vp, _P], _i32),
    "cr_concat_key_slices": ([_P, _u32, _vp, _P], _i32),
    "cr_upload_portable_ex": ([_vp, _u64, _u32, _vp, _u32, _u32, _P], _i32),
    "cr_portable_meta": ([_vp, _u64, _vp], _i32),
    "cr_topk_comm_unique_id": ([_vp, _u32], _i32),
    "cr_topk_comm_init": ([_vp, _i32, _i32, C.POINTER(_vp)], _i32),
    "cr_topk_comm_size": ([_vp, C.POINTER(_i32), C.POINTER(_i32)], _i32),
    "cr_topk_comm_destroy": ([_vp], _i32),
    "cr_filtered_topk_sharded": ([_vp, _i32, _vp, _vp, _u64, _u32, _vp, _u32, _P, _u64, _u32, _i32, _vp, _vp,
                                  _vp], _i32),
}
for _name, (_args, _res) in _sigs.items():
    _f = getattr(_lib, _name)
    _f.argtypes = _args
    _f.restype = _res


def lib() -> C.CDLL:
    return _lib


def version() -> str:
    return _lib.cr_version().decode()


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {_lib.cr_last_error_string().decode()}")


def _torch():
    import torch  # plumbing for device memory and streams

    return torch


def _stream_ptr(stream) -> int | None:
    if stream is None or stream == 0:
        return None
    return int(getattr(stream, "cuda_stream", stream)) or None


def _dev_ptr(t) -> int:
    return int(t.data_ptr())


class GpuRoaring:
    """Owner of one device bitmap; `.raw` is the C struct, `.free()` releases it."""

    def __init__(self, raw: CrGpuRoaring | None = None):
        self.raw = raw if raw is not None else CrGpuRoaring()

    def __getattr__(self, name):
        raw = object.__getattribute__(self, "raw")
        return getattr(raw, name)

    @property
    def negated_flag(self) -> bool:
        return bool(self.raw.negated)

    def free(self, stream=None) -> None:
        if stream is None:
            _check(_lib.cr_gpu_roaring_free(C.byref(self.raw)), "gpu_roaring_free")
        else:
            _check(_lib.cr_gpu_roaring_free_async(C.byref(self.raw), _stream_ptr(stream)),
                   "gpu_roaring_free_async")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.free()

    def image(self) -> dict:
        """Host copy of the packed layout (for parity checks)."""
        torch = _torch()
        torch.cuda.synchronize()
        r = self.raw
        n = r.n_containers

        def dl(ptr, count, dtype):
            out = np.zeros(count, dtype=dtype)
            if count and ptr:
                _memcpy_d2h(out, ptr)
            return out

        return {
            "n_containers": n, "universe_size": r.universe_size,
            "total_cardinality": r.total_cardinality, "negated": bool(r.negated),
            "n_bitmap": r.n_bitmap_containers, "n_array": r.n_array_containers,
            "n_run": r.n_run_containers, "array_pool_bytes": r.array_pool_bytes,
            "run_pool_bytes": r.run_pool_bytes, "max_key": r.max_key if n else 0,
            "keys": dl(r.keys, n, np.uint16), "types": dl(r.types, n, np.uint8),
            "offsets": dl(r.offsets, n, np.uint32), "cards": dl(r.cardinalities, n, np.uint16),
            "key_index": dl(r.key_index, (r.max_key + 1) if (n and r.key_index) else 0, np.uint16),
            "bitmap": dl(r.bitmap_data, r.n_bitmap_containers * 1024, np.uint64),
            "array": dl(r.array_data, r.array_pool_bytes // 2, np.uint16),
            "run": dl(r.run_data, r.run_pool_bytes // 2, np.uint16),
        }


_cudart = None


def _memcpy_d2h(out: np.ndarray, ptr: int) -> None:
    global _cudart
    if _cudart is None:
        _cudart = C.CDLL("libcudart.so.12") if _has("libcudart.so.12") else C.CDLL("libcudart.so")
        _cudart.cudaMemcpy.argtypes = [_vp, _vp, C.c_size_t, C.c_int]
        _cudart.cudaMemcpy.restype = C.c_int
    rc = _cudart.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy D2H failed ({rc})")


def _has(name: str) -> bool:
    try:
        C.CDLL(name)
        return True
    except OSError:
        return False


# ------------------------------------------------------------------ construction

def upload_from_ids(ids, universe_size: int, stream=None, bitmap_threshold: int = PROMOTE_AUTO) -> GpuRoaring:
    """reference upload_from_ids (src/upload_ids.cu:567). `ids`: host numpy
    uint32 array, or a CUDA uint32/int32 tensor (device path)."""
    out = GpuRoaring()
    if isinstance(ids, np.ndarray):
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        rc = _lib.cr_upload_from_ids(a.ctypes.data if a.size else None, a.size, universe_size,
                                     _stream_ptr(stream), bitmap_threshold, C.byref(out.raw))
    else:
        rc = _lib.cr_upload_from_device_ids(_dev_ptr(ids) if ids.numel() else None, ids.numel(),
                                            universe_size, _stream_ptr(stream), bitmap_threshold,
                                            C.byref(out.raw))
    _check(rc, "upload_from_ids")
    return out


upload_from_sorted_ids = upload_from_ids


def upload_from_bitset(words, universe_size: int, stream=None, bitmap_threshold: int = PROMOTE_AUTO) -> GpuRoaring:
    out = GpuRoaring()
    a = np.ascontiguousarray(words, dtype=np.uint32)
    _check(_lib.cr_upload_from_bitset(a.ctypes.data if a.size else None, a.size, universe_size,
                                      _stream_ptr(stream), bitmap_threshold, C.byref(out.raw)),
           "upload_from_bitset")
    return out


def upload_from_device_bitset(words, universe_size: int, stream=None,
                              bitmap_threshold: int = PROMOTE_AUTO) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_upload_from_device_bitset(_dev_ptr(words) if words.numel() else None, words.numel(),
                                             universe_size, _stream_ptr(stream), bitmap_threshold,
                                             C.byref(out.raw)), "upload_from_device_bitset")
    return out


PORTABLE_KEEP_UNCOMPLEMENTED = 1


def upload_portable(data: bytes, universe_size: int, stream=None, bitmap_threshold: int = PROMOTE_AUTO,
                    flags: int = 0) -> GpuRoaring:
    """A bitmap in the portable Roaring serialization (bytes) -> GpuRoaring.
    flags=PORTABLE_KEEP_UNCOMPLEMENTED never stores the complement."""
    out = GpuRoaring()
    buf = C.create_string_buffer(bytes(data), len(data)) if len(data) else None
    _check(_lib.cr_upload_portable_ex(C.cast(buf, C.c_void_p) if buf is not None else None, len(data),
                                      universe_size, _stream_ptr(stream), bitmap_threshold, flags,
                                      C.byref(out.raw)), "upload_portable")
    return out


class CrRoaringMeta(C.Structure):
    _fields_ = [("n_containers", C.c_uint32), ("n_bitmap_containers", C.c_uint32),
                ("n_array_containers", C.c_uint32), ("n_run_containers", C.c_uint32),
                ("universe_size", C.c_uint32), ("max_key", C.c_uint32), ("total_bytes", C.c_uint64),
                ("total_cardinality", C.c_uint64)]


def portable_meta(data: bytes) -> dict:
    """Container counts and device footprint of a portable serialization
    (host only; the reference's get_meta(const roaring_bitmap_t*))."""
    m = CrRoaringMeta()
    buf = C.create_string_buffer(bytes(data), len(data)) if len(data) else None
    _check(_lib.cr_portable_meta(C.cast(buf, C.c_void_p) if buf is not None else None, len(data), C.byref(m)),
           "portable_meta")
    return {f: getattr(m, f) for f, _ in CrRoaringMeta._fields_}


class CrRoaringBatch(C.Structure):
    """Layout of cr_roaring_batch / cu_roaring::v2::GpuRoaringBatch."""
    _fields_ = [("n_bitmaps", C.c_uint32), ("total_containers", C.c_uint32),
                ("n_bitmap_containers_total", C.c_uint32), ("array_pool_bytes", C.c_uint32),
                ("run_pool_bytes", C.c_uint32), ("container_starts", C.c_void_p), ("key_index_starts", C.c_void_p),
                ("keys", C.c_void_p), ("types", C.c_void_p), ("offsets", C.c_void_p),
                ("cardinalities", C.c_void_p), ("key_indices", C.c_void_p), ("bitmap_data", C.c_void_p),
                ("array_data", C.c_void_p), ("run_data", C.c_void_p),
                ("host_total_cardinalities", C.POINTER(C.c_uint64)),
                ("host_universe_sizes", C.POINTER(C.c_uint32)),
                ("host_container_starts", C.POINTER(C.c_uint32)),
                ("host_key_index_starts", C.POINTER(C.c_uint32)),
                ("host_n_bitmap_containers", C.POINTER(C.c_uint32)),
                ("_alloc_base", C.c_void_p), ("_host_meta_base", C.c_void_p)]


class RoaringBatch:
    """N bitmaps in one device block (the reference's v2 GpuRoaringBatch)."""

    def __init__(self, raw: CrRoaringBatch | None = None):
        self.raw = raw if raw is not None else CrRoaringBatch()

    @property
    def n_bitmaps(self) -> int:
        return self.raw.n_bitmaps

    def total_cardinality(self, b: int) -> int:
        return int(self.raw.host_total_cardinalities[b])

    def universe_size(self, b: int) -> int:
        return int(self.raw.host_universe_sizes[b])

    def free(self) -> None:
        _check(_lib.cr_batch_free(C.byref(self.raw)), "batch_free")

    def promote(self, stream=None) -> "RoaringBatch":
        out = RoaringBatch()
        _check(_lib.cr_batch_promote(C.byref(self.raw), _stream_ptr(stream), C.byref(out.raw)), "batch_promote")
        return out

    def multi_and(self, indices, stream=None) -> "RoaringBatch":
        idx = (C.c_uint32 * len(indices))(*indices)
        out = RoaringBatch()
        _check(_lib.cr_batch_multi_and(C.byref(self.raw), idx, len(indices), _stream_ptr(stream), C.byref(out.raw)),
               "batch_multi_and")
        return out

    def decompress(self, words_each: int, stream=None):
        """[n_bitmaps, words_each] int64 (u64 words) on the device, zeroed first."""
        torch = _torch()
        out = torch.zeros((max(1, self.n_bitmaps), words_each), dtype=torch.int64, device="cuda")
        _check(_lib.cr_batch_decompress(C.byref(self.raw), _dev_ptr(out), words_each, _stream_ptr(stream)),
               "batch_decompress")
        return out

    def contains(self, bitmap_idx, ids, stream=None):
        """bool[n]: contains(batch, bitmap_idx[i], ids[i]) (device int32 tensors)."""
        torch = _torch()
        n = ids.numel()
        bits = torch.zeros(((n + 31) // 32,), dtype=torch.int32, device="cuda")
        _check(_lib.cr_batch_contains(C.byref(self.raw), _dev_ptr(bitmap_idx), _dev_ptr(ids), n, _dev_ptr(bits),
                                      _stream_ptr(stream)), "batch_contains")
        shifts = torch.arange(32, device="cuda", dtype=torch.int32)
        return ((bits[:, None] >> shifts[None, :]) & 1).flatten()[:n].bool()


def batch_upload_portable(buffers, stream=None) -> RoaringBatch:
    """Bitmaps in the portable Roaring serialization (list of bytes) -> a batch."""
    n = len(buffers)
    keep = [C.create_string_buffer(bytes(b), len(b)) for b in buffers]
    ptrs = (C.c_void_p * max(1, n))(*[C.cast(k, C.c_void_p) for k in keep])
    sizes = (C.c_uint64 * max(1, n))(*[len(b) for b in buffers])
    out = RoaringBatch()
    _check(_lib.cr_batch_upload_portable(ptrs, sizes, n, _stream_ptr(stream), C.byref(out.raw)),
           "batch_upload_portable")
    return out


def gpu_roaring_free(bm: GpuRoaring) -> None:
    bm.free()


def gpu_roaring_free_async(bm: GpuRoaring, stream) -> None:
    bm.free(stream if stream is not None else 0)


# --------------------------------------------------------------------- promotion

def resolve_auto_threshold(universe_size: int, device_id: int = -1) -> int:
    v = C.c_uint32()
    _check(_lib.cr_resolve_auto_threshold(universe_size, device_id, C.byref(v)), "resolve_auto_threshold")
    return v.value


def promote_to_bitmap(bm: GpuRoaring, stream=None) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_promote_to_bitmap(C.byref(bm.raw), _stream_ptr(stream), C.byref(out.raw)),
           "promote_to_bitmap")
    return out


def promote_auto(bm: GpuRoaring, stream=None, device_id: int = -1) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_promote_auto(C.byref(bm.raw), _stream_ptr(stream), device_id, C.byref(out.raw)),
           "promote_auto")
    return out


def gpu_roaring_deep_copy(bm: GpuRoaring, stream=None) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_deep_copy(C.byref(bm.raw), _stream_ptr(stream), C.byref(out.raw)), "deep_copy")
    return out


# ------------------------------------------------------------------- set algebra

def set_operation(a: GpuRoaring, b: GpuRoaring, op: int, stream=None) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_set_operation(C.byref(a.raw), C.byref(b.raw), op, _stream_ptr(stream),
                                 C.byref(out.raw)), "set_operation")
    return out


def _array_of(bms):
    arr = (CrGpuRoaring * max(1, len(bms)))()
    for i, b in enumerate(bms):
        arr[i] = b.raw
    return arr


def multi_and(bms, stream=None) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_multi_and(_array_of(bms), len(bms), _stream_ptr(stream), C.byref(out.raw)), "multi_and")
    return out


def multi_or(bms, stream=None) -> GpuRoaring:
    out = GpuRoaring()
    _check(_lib.cr_multi_or(_array_of(bms), len(bms), _stream_ptr(stream), C.byref(out.raw)), "multi_or")
    return out


# ------------------------------------------------------------------------ export

def decompress_to_bitset(bm: GpuRoaring, output=None, stream=None):
    """Returns (or fills) a CUDA int32 tensor of ceil(U/32) words."""
    torch = _torch()
    if output is None:
        output = torch.empty(max(1, (bm.raw.universe_size + 31) // 32), dtype=torch.int32, device="cuda")
        n = (bm.raw.universe_size + 31) // 32
    else:
        n = output.numel()
    _check(_lib.cr_decompress_to_bitset(C.byref(bm.raw), _dev_ptr(output), n, _stream_ptr(stream)),
           "decompress_to_bitset")
    return output[:n] if n else output[:0]


def enumerate_ids(bm: GpuRoaring, output=None, stream=None, dtype="int64"):
    """Sorted IDs of the logical set as a CUDA tensor (int64, or int32 for u32)."""
    torch = _torch()
    n = int(bm.raw.total_cardinality)
    tdt = torch.int64 if dtype == "int64" else torch.int32
    if output is None:
        output = torch.empty(max(1, n), dtype=tdt, device="cuda")
    fn = _lib.cr_enumerate_ids_i64 if tdt == torch.int64 else _lib.cr_enumerate_ids_u32
    _check(fn(C.byref(bm.raw), _dev_ptr(output), _stream_ptr(stream)), "enumerate_ids")
    return output[:n]


to_csr = enumerate_ids


def contains_batch(bm: GpuRoaring, ids, out_bits=None, warp: bool = False, stream=None):
    """Bit i of the returned int32 words = contains(ids[i]) (CUDA tensors)."""
    torch = _torch()
    n = ids.numel()
    if out_bits is None:
        out_bits = torch.empty(max(1, (n + 31) // 32), dtype=torch.int32, device="cuda")
    _check(_lib.cr_contains_batch(C.byref(bm.raw), _dev_ptr(ids), n, _dev_ptr(out_bits), int(warp),
                                  _stream_ptr(stream)), "contains_batch")
    return out_bits


# ------------------------------------------------------------- filtered top-k

def row_norms(db, stream=None):
    torch = _torch()
    out = torch.empty(db.shape[0], dtype=torch.float32, device=db.device)
    _check(_lib.cr_row_norms(_dev_ptr(db), db.shape[0], db.shape[1], _dev_ptr(out), _stream_ptr(stream)),
           "row_norms")
    return out


def filtered_topk(db, queries, k: int, metric: int = METRIC_IP, filter: GpuRoaring | None = None,
                  db_norms=None, row_offset: int = 0, stream=None, out_dist=None, out_ids=None):
    """Exact filtered top-k (fp16 db/queries, fp32 accumulate). Returns (dist, ids)."""
    torch = _torch()
    q = queries.shape[0]
    if out_dist is None:
        out_dist = torch.empty((q, k), dtype=torch.float32, device=db.device)
    if out_ids is None:
        out_ids = torch.empty((q, k), dtype=torch.int64, device=db.device)
    _check(_lib.cr_filtered_topk(_dev_ptr(db), _dev_ptr(db_norms) if db_norms is not None else None,
                                 db.shape[0], db.shape[1], _dev_ptr(queries), q,
                                 C.byref(filter.raw) if filter is not None else None, row_offset, k,
                                 metric, _dev_ptr(out_dist), _dev_ptr(out_ids), _stream_ptr(stream)),
           "filtered_topk")
    return out_dist, out_ids


def topk_merge(dist_parts, id_parts, k: int, metric: int = METRIC_IP, stream=None):
    torch = _torch()
    p, q, _ = dist_parts.shape
    out_d = torch.empty((q, k), dtype=torch.float32, device=dist_parts.device)
    out_i = torch.empty((q, k), dtype=torch.int64, device=dist_parts.device)
    _check(_lib.cr_topk_merge(_dev_ptr(dist_parts), _dev_ptr(id_parts), p, q, k, metric, _dev_ptr(out_d),
                              _dev_ptr(out_i), _stream_ptr(stream)), "topk_merge")
    return out_d, out_i


def topk_packed_buffer(n_queries: int, k: int, device):
    """A send block for one shard's top-k: (block, dist view, ids view). Pass
    the views as filtered_topk's out_dist / out_ids, gather the blocks with one
    collective, and merge them with topk_merge_packed."""
    torch = _torch()
    if (n_queries * k) % 2:
        raise ValueError("n_queries * k must be even for the packed layout")
    nd = n_queries * k
    block = torch.empty(nd * 12, dtype=torch.uint8, device=device)
    dist = block[: nd * 4].view(torch.float32).view(n_queries, k)
    ids = block[nd * 4:].view(torch.int64).view(n_queries, k)
    return block, dist, ids


def topk_merge_packed(blocks, n_queries: int, k: int, metric: int = METRIC_IP, stream=None):
    """Merge [parts, 12 * n_queries * k] uint8 blocks (see topk_packed_buffer)."""
    torch = _torch()
    p = blocks.shape[0]
    out_d = torch.empty((n_queries, k), dtype=torch.float32, device=blocks.device)
    out_i = torch.empty((n_queries, k), dtype=torch.int64, device=blocks.device)
    _check(_lib.cr_topk_merge_packed(_dev_ptr(blocks), blocks.stride(0), p, n_queries, k, metric,
                                     _dev_ptr(out_d), _dev_ptr(out_i), _stream_ptr(stream)), "topk_merge_packed")
    return out_d, out_i


# ------------------------------------------------- row-sharded top-k (NCCL)

TOPK_COMM_ID_BYTES = 128


def topk_comm_unique_id() -> bytes:
    """Rank 0 makes the communicator's id; hand it to every rank."""
    buf = C.create_string_buffer(TOPK_COMM_ID_BYTES)
    _check(_lib.cr_topk_comm_unique_id(buf, TOPK_COMM_ID_BYTES), "topk_comm_unique_id")
    return buf.raw


class TopkComm:
    """The communicator of cr_filtered_topk_sharded (one per rank; every
    rank constructs it together, with its own GPU current)."""

    def __init__(self, unique_id: bytes, n_ranks: int, rank: int):
        if len(unique_id) != TOPK_COMM_ID_BYTES:
            raise ValueError("unique_id must be TOPK_COMM_ID_BYTES bytes")
        self.handle = C.c_void_p()
        _check(_lib.cr_topk_comm_init(C.c_char_p(unique_id), n_ranks, rank, C.byref(self.handle)),
               "topk_comm_init")
        self.n_ranks, self.rank = n_ranks, rank

    def destroy(self) -> None:
        if self.handle:
            _check(_lib.cr_topk_comm_destroy(self.handle), "topk_comm_destroy")
            self.handle = C.c_void_p()


def filtered_topk_sharded(comm: TopkComm, db, queries, k: int, metric: int = METRIC_IP,
                          filter: GpuRoaring | None = None, db_norms=None, row_offset: int = 0, root: int = 0,
                          stream=None, out_dist=None, out_ids=None):
    """This rank's rows `db` (global row IDs from row_offset) searched and the
    per-rank lists merged on `root`. Returns (dist, ids) on the root, None
    elsewhere."""
    torch = _torch()
    q = queries.shape[0]
    is_root = comm.rank == root
    if is_root and out_dist is None:
        out_dist = torch.empty((q, k), dtype=torch.float32, device=db.device)
    if is_root and out_ids is None:
        out_ids = torch.empty((q, k), dtype=torch.int64, device=db.device)
    _check(_lib.cr_filtered_topk_sharded(
        comm.handle, root, _dev_ptr(db), _dev_ptr(db_norms) if db_norms is not None else None, db.shape[0],
        db.shape[1], _dev_ptr(queries), q, C.byref(filter.raw) if filter is not None else None, row_offset, k,
        metric, _dev_ptr(out_dist) if is_root else None, _dev_ptr(out_ids) if is_root else None,
        _stream_ptr(stream)), "filtered_topk_sharded")
    return (out_dist, out_ids) if is_root else None


# ------------------------------------------------------------- measurement

(KERNEL_TOPK, KERNEL_CONTAINS, KERNEL_SETOP, KERNEL_UPLOAD_SCATTER, KERNEL_UPLOAD_EMIT, KERNEL_DECOMPRESS,
 KERNEL_TOPK_MERGE, KERNEL_TOPK_COMPACT) = range(8)


def profile_enable(on: bool = True) -> None:
    _lib.cr_profile_enable(int(on))


def profile_kinds(*kernels: int) -> None:
    """Bracket only these kernel ids while profiling is on (none given: all)."""
    mask = 0xFFFFFFFF if not kernels else sum(1 << k for k in set(kernels))
    _lib.cr_profile_kinds(mask)


def profile_mean_ms(kernel: int) -> tuple[float, int]:
    """Mean device time of the profiled launches of `kernel` since profiling
    was switched on, and their number (0.0, 0 when none)."""
    tot, n = C.c_float(), C.c_uint32()
    _check(_lib.cr_profile_sum_ms(kernel, C.byref(tot), C.byref(n)), "profile_sum_ms")
    return (tot.value / n.value if n.value else 0.0), n.value


def profile_last_ms(kernel: int) -> float:
    v = C.c_float()
    _check(_lib.cr_profile_last_ms(kernel, C.byref(v)), "profile_last_ms")
    return v.value


# ------------------------------------------------------------- sharding

def key_range(universe_size: int, rank: int, world: int) -> tuple[int, int]:
    """Rank `rank`'s container keys [lo, hi) when a bitmap over universe_size
    is split at chunk (65536-ID) boundaries over `world` ranks."""
    lo, hi = C.c_uint32(), C.c_uint32()
    _check(_lib.cr_key_range(universe_size, rank, world, C.byref(lo), C.byref(hi)), "key_range")
    return lo.value, hi.value


def key_slice(bm: GpuRoaring, key_lo: int, key_hi: int, stream=None) -> GpuRoaring:
    """The containers of `bm` with keys in [key_lo, key_hi), as a new bitmap."""
    out = GpuRoaring()
    _check(_lib.cr_key_slice(C.byref(bm.raw), key_lo, key_hi, _stream_ptr(stream), C.byref(out.raw)), "key_slice")
    return out


def concat_key_slices(slices, stream=None) -> GpuRoaring:
    """Slices with ascending, disjoint key ranges laid end to end."""
    out = GpuRoaring()
    arr = (CrGpuRoaring * max(1, len(slices)))(*[b.raw for b in slices])
    _check(_lib.cr_concat_key_slices(arr, len(slices), _stream_ptr(stream), C.byref(out.raw)), "concat_key_slices")
    return out


def shard_range(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row range [lo, hi) of `rank` when n_rows are split over
    `world` ranks (the filtered top-k shards the database this way; row IDs
    stay global via row_offset = lo)."""
    return n_rows * rank // world, n_rows * (rank + 1) // world
