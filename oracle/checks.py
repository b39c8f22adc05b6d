"""Parity checks shared by tests/ and bench.py's parity legs.

TEST INFRASTRUCTURE ONLY: these helpers compare the engine's outputs with
the CPU oracle (roaring_oracle.c) or with a plain PyTorch fp32 computation;
nothing in the product path imports them, and bench.py calls them only
outside its timed regions.
"""
from __future__ import annotations

import numpy as np

# Distances within 1e-3 relative; id sets equal except
# where the reference's k-th distance ties within that tolerance.
TOPK_RTOL = 1e-3


class ParityError(AssertionError):
    pass


def _require(cond, msg):
    if not cond:
        raise ParityError(msg)


def assert_same_image(dev_image: dict, ora_image: dict, what: str = "") -> None:
    """Bit-exact comparison of two packed images (GpuRoaring.image() /
    OracleBitmap.image()): counts, flags, metadata arrays and the pools."""
    for k in ("n_containers", "universe_size", "total_cardinality", "negated", "n_bitmap", "n_array",
              "n_run", "array_pool_bytes", "run_pool_bytes", "max_key"):
        _require(dev_image[k] == ora_image[k], f"{what}: field {k}: gpu {dev_image[k]} != oracle {ora_image[k]}")
    for k in ("keys", "types", "offsets", "cards", "key_index", "bitmap", "array", "run"):
        _require(np.array_equal(dev_image[k], ora_image[k]), f"{what}: array {k} differs")


def check_topk(d_gpu, i_gpu, d_ref, i_ref, what: str = "") -> None:
    """Distances within TOPK_RTOL relative; id sets equal up to ties at the
    k-th distance (within the same tolerance)."""
    d_gpu, i_gpu, d_ref, i_ref = (np.asarray(x) for x in (d_gpu, i_gpu, d_ref, i_ref))
    valid = i_ref >= 0
    _require(np.array_equal(valid, i_gpu >= 0), f"{what}: number of results differs")
    scale = np.maximum(np.abs(d_ref), 1e-3)
    diff = np.abs(np.where(valid, d_gpu - d_ref, 0.0))
    _require(bool((diff <= TOPK_RTOL * scale + 1e-6).all()), f"{what}: max distance error {diff.max()}")
    for qi in range(d_ref.shape[0]):
        a = set(i_gpu[qi][valid[qi]].tolist())
        b = set(i_ref[qi][valid[qi]].tolist())
        if a == b:
            continue
        kth = d_ref[qi][valid[qi]][-1]
        for r in a ^ b:
            pos = np.flatnonzero(i_gpu[qi] == r)
            dist = d_gpu[qi][pos[0]] if pos.size else d_ref[qi][np.flatnonzero(i_ref[qi] == r)[0]]
            _require(abs(dist - kth) <= TOPK_RTOL * max(abs(kth), 1e-3) + 1e-6,
                     f"{what}: query {qi}: id {r} differs away from the k-th distance")


def torch_exact_topk(torch, db, queries, k: int, metric: int, mask=None, row_offset: int = 0, chunk: int = 1 << 20):
    """Exact fp32 filtered top-k with torch on the GPU (fp16 inputs widened
    to fp32, rows outside `mask` excluded, ties to the smaller id). Returns
    (dist [Q, k] fp32, ids [Q, k] int64 global, -1 where fewer pass); IP
    distances are scores (larger first), L2 squared distances (smaller
    first)."""
    q = queries.float()
    nq = q.shape[0]
    best_s = torch.full((nq, k), -float("inf"), device=db.device)
    best_i = torch.full((nq, k), -1, dtype=torch.int64, device=db.device)
    qn = (q * q).sum(1, keepdim=True)
    for lo in range(0, db.shape[0], chunk):
        x = db[lo:lo + chunk].float()
        s = q @ x.T
        if metric == 1:  # larger is better internally: -(|q|^2 - 2 q.x + |x|^2)
            s = 2 * s - (x * x).sum(1)[None, :] - qn
        if mask is not None:
            s = torch.where(mask[lo:lo + chunk][None, :], s, torch.full_like(s, -float("inf")))
        ids = torch.arange(lo, lo + x.shape[0], device=db.device, dtype=torch.int64) + row_offset
        cs = torch.cat([best_s, s], 1)
        ci = torch.cat([best_i, ids[None, :].expand(nq, -1)], 1)
        # Stable order: score descending, then id ascending (ids of a chunk
        # only grow, so a stable sort on the score keeps ties in id order).
        order = torch.sort(cs, dim=1, descending=True, stable=True).indices[:, :k]
        best_s = torch.gather(cs, 1, order)
        best_i = torch.gather(ci, 1, order)
    best_i = torch.where(torch.isinf(best_s), torch.full_like(best_i, -1), best_i)
    d = -best_s if metric == 1 else best_s
    return d, best_i


def merge_exact(parts_d, parts_i, k: int, metric: int):
    """Merge per-shard exact lists (numpy) into one [Q, k] list."""
    d = np.concatenate(parts_d, 1)
    i = np.concatenate(parts_i, 1)
    key = np.where(i < 0, np.inf, -d if metric == 0 else d)
    order = np.lexsort((np.where(i < 0, np.iinfo(np.int64).max, i), key), axis=1)[:, :k]
    return np.take_along_axis(d, order, 1), np.take_along_axis(i, order, 1)
