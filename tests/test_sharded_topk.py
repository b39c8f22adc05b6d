"""cr_filtered_topk_sharded: the row-sharded search with the NCCL gather and
the root's merge inside the library.

CPU: NCCL resolves at run time and hands out a communicator id (no GPU work).
GPU: a one-rank communicator gives exactly cr_filtered_topk's answer; with two
or more visible GPUs, two processes (one per GPU) each search half of the rows
and the root's merged answer matches the exact CPU oracle.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest


def test_nccl_resolves_and_makes_an_id(built_lib):
    # The library binds to the NCCL the process has already loaded and only
    # otherwise opens libnccl.so.2 from the search path. PyTorch ships its own
    # (newer) copy under the same soname, so a process that uses both loads
    # torch first, as every user of these bindings does.
    import torch  # noqa: F401

    lib = C.CDLL(str(built_lib))
    buf = C.create_string_buffer(128)
    rc = lib.cr_topk_comm_unique_id(buf, 128)
    if rc == -6:  # CR_ERR_UNSUPPORTED: no NCCL on this host
        pytest.skip("NCCL is not installed")
    assert rc == 0
    assert any(buf.raw)
    assert lib.cr_topk_comm_unique_id(buf, 16) == -1  # too small a buffer


def _data(n, q, seed):
    rng = np.random.default_rng(seed)
    db = rng.standard_normal((n, 128)).astype(np.float32)
    db /= np.linalg.norm(db, axis=1, keepdims=True)
    qs = rng.standard_normal((q, 128)).astype(np.float32)
    qs /= np.linalg.norm(qs, axis=1, keepdims=True)
    keep = np.flatnonzero(rng.random(n) < 0.2).astype(np.uint32)
    return db.astype(np.float16), qs.astype(np.float16), keep


@pytest.mark.gpu
@pytest.mark.parametrize("metric", [0, 1])
def test_one_rank_equals_filtered_topk(cr, metric):
    import torch

    db, qs, keep = _data(50_000, 70, seed=metric)
    filt = cr.upload_from_ids(keep, 50_000)
    comm = cr.TopkComm(cr.topk_comm_unique_id(), 1, 0)
    try:
        ddb, dq = torch.from_numpy(db).cuda(), torch.from_numpy(qs).cuda()
        norms = cr.row_norms(ddb) if metric == 1 else None
        d0, i0 = cr.filtered_topk(ddb, dq, 30, metric=metric, filter=filt, db_norms=norms)
        d1, i1 = cr.filtered_topk_sharded(comm, ddb, dq, 30, metric=metric, filter=filt, db_norms=norms)
        assert torch.equal(i0, i1) and torch.equal(d0, d1)
    finally:
        comm.destroy()
        filt.free()


def _rank_main(rank, world, uid, n, q, k, metric, out_path):
    import torch

    import cu_roaring_b200 as cr

    torch.cuda.set_device(rank)
    db, qs, keep = _data(n, q, seed=5)
    lo, hi = cr.shard_range(n, rank, world)
    filt = cr.upload_from_ids(keep, n)
    comm = cr.TopkComm(uid, world, rank)
    ddb = torch.from_numpy(np.ascontiguousarray(db[lo:hi])).cuda()
    dq = torch.from_numpy(qs).cuda()
    norms = cr.row_norms(ddb) if metric == 1 else None
    res = None
    for _ in range(3):  # repeated calls reuse the gather buffer
        res = cr.filtered_topk_sharded(comm, ddb, dq, k, metric=metric, filter=filt, db_norms=norms, row_offset=lo,
                                       root=0)
    torch.cuda.synchronize()
    if rank == 0:
        np.savez(out_path, d=res[0].cpu().numpy(), i=res[1].cpu().numpy())
    comm.destroy()
    filt.free()


@pytest.mark.gpu
@pytest.mark.parametrize("metric", [0, 1])
def test_two_ranks_match_oracle(cr, oracle, tmp_path, metric):
    import torch
    import torch.multiprocessing as mp

    from checks import check_topk

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, n, q, k = 2, 90_001, 48, 40
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    uid = cr.topk_comm_unique_id()
    out = tmp_path / "root.npz"
    mp.start_processes(_rank_main, args=(world, uid, n, q, k, metric, str(out)), nprocs=world, join=True,
                       start_method="spawn")
    got = np.load(out)
    db, qs, keep = _data(n, q, seed=5)
    words = np.zeros((n + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(words, keep // 32, (1 << (keep % 32)).astype(np.uint32))
    d_ref, i_ref = oracle.topk(db, qs, k, metric, words)
    check_topk(got["d"], got["i"], d_ref, i_ref, "two ranks")
