"""CPU, two gloo ranks: the multi-GPU top-k exchange without a GPU.

Each rank takes its row range (cu_roaring_b200.shard_range), computes the
exact filtered top-k of its shard with GLOBAL row ids (the CPU oracle stands
in for cr_filtered_topk with row_offset), the per-rank [Q x k] lists are
all_gathered (gloo here, NCCL in bench.py), and rank 0 merges them with the
library's ordering rule (better score, then smaller id). The result must equal
the unsharded search.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(n=6000, q=9, dim=128, seed=3):
    rng = np.random.default_rng(seed)
    db = rng.standard_normal((n, dim)).astype(np.float32)
    db /= np.linalg.norm(db, axis=1, keepdims=True)
    qs = rng.standard_normal((q, dim)).astype(np.float32)
    qs /= np.linalg.norm(qs, axis=1, keepdims=True)
    keep = rng.random(n) < 0.3
    return db.astype(np.float16), qs.astype(np.float16), keep


def _words(mask):
    w = np.zeros((mask.size + 31) // 32, dtype=np.uint32)
    idx = np.flatnonzero(mask)
    np.bitwise_or.at(w, idx // 32, (1 << (idx % 32)).astype(np.uint32))
    return w


def merge_lists(dist_parts, id_parts, k, metric):
    """Host restatement of cr_topk_merge's ordering: best score first, ties to
    the smaller id, missing entries (id -1) last."""
    out_d = np.zeros((dist_parts.shape[1], k), np.float32)
    out_i = np.zeros((dist_parts.shape[1], k), np.int64)
    for qi in range(dist_parts.shape[1]):
        cand = [(d, i) for p in range(dist_parts.shape[0])
                for d, i in zip(dist_parts[p, qi], id_parts[p, qi]) if i >= 0]
        cand.sort(key=lambda t: ((-t[0]) if metric == 0 else t[0], t[1]))
        cand = cand[:k] + [((-np.inf if metric == 0 else np.inf), -1)] * (k - len(cand))
        out_d[qi] = [c[0] for c in cand]
        out_i[qi] = [c[1] for c in cand]
    return out_d, out_i


def _worker(rank, world, port, k, metric, result_path):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "cu-roaring-bitmap_b200", repo / "oracle"):
        sys.path.insert(0, str(p))
    import oracle
    from cu_roaring_b200 import shard_range  # noqa: E402  (pure host helper)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    db, qs, keep = _data()
    lo, hi = shard_range(db.shape[0], rank, world)
    d, i = oracle.topk(db[lo:hi], qs, k, metric, _words(keep[lo:hi]))
    i = np.where(i >= 0, i + lo, -1)
    gd = [torch.zeros((qs.shape[0], k)) for _ in range(world)]
    gi = [torch.zeros((qs.shape[0], k), dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gd, torch.from_numpy(d))
    dist.all_gather(gi, torch.from_numpy(i))
    if rank == 0:
        md, mi = merge_lists(torch.stack(gd).numpy(), torch.stack(gi).numpy(), k, metric)
        np.savez(result_path, d=md, i=mi)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("metric", [0, 1])
def test_two_rank_sharded_topk_equals_unsharded(tmp_path, metric, built_lib):
    pytest.importorskip("torch.distributed")
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "oracle"))
    import oracle

    if "cu_roaring_b200" not in sys.modules:
        # the helper lives in the package; the package needs the built .so
        pytest.importorskip("cu_roaring_b200")
    k, world = 20, 2
    out = tmp_path / "merged.npz"
    mp.spawn(_worker, args=(world, _free_port(), k, metric, str(out)), nprocs=world, join=True)
    got = np.load(out)
    db, qs, keep = _data()
    want_d, want_i = oracle.topk(db, qs, k, metric, _words(keep))
    assert np.array_equal(got["i"], want_i)
    np.testing.assert_allclose(got["d"], want_d, rtol=1e-5)


def _packed_worker(rank, world, port, k, metric, result_path):
    """Each rank writes its shard's top-k into the packed send block (fp32
    distances, then int64 ids), gathers the blocks to rank 0 in one
    collective, and rank 0 reads the views back out of the gathered bytes:
    the same exchange bench.py runs over NCCL, here over gloo."""
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "cu-roaring-bitmap_b200", repo / "oracle"):
        sys.path.insert(0, str(p))
    import oracle
    from cu_roaring_b200 import shard_range, topk_packed_buffer  # noqa: E402

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    db, qs, keep = _data()
    nq = qs.shape[0]
    lo, hi = shard_range(db.shape[0], rank, world)
    d, i = oracle.topk(db[lo:hi], qs, k, metric, _words(keep[lo:hi]))
    block, bd, bi = topk_packed_buffer(nq, k, "cpu")
    bd.copy_(torch.from_numpy(d))
    bi.copy_(torch.from_numpy(np.where(i >= 0, i + lo, -1)))
    gathered = torch.empty((world, block.numel()), dtype=torch.uint8)
    dist.gather(block, gather_list=list(gathered.unbind(0)) if rank == 0 else None, dst=0)
    if rank == 0:
        nd = nq * k
        gd = gathered[:, : nd * 4].contiguous().view(torch.float32).view(world, nq, k)
        gi = gathered[:, nd * 4:].contiguous().view(torch.int64).view(world, nq, k)
        md, mi = merge_lists(gd.numpy(), gi.numpy(), k, metric)
        np.savez(result_path, d=md, i=mi)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("metric", [0, 1])
def test_two_rank_packed_gather_equals_unsharded(tmp_path, metric, built_lib):
    pytest.importorskip("torch.distributed")
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "oracle"))
    import oracle

    if "cu_roaring_b200" not in sys.modules:
        pytest.importorskip("cu_roaring_b200")
    k, world = 20, 2
    out = tmp_path / "merged.npz"
    mp.spawn(_packed_worker, args=(world, _free_port(), k, metric, str(out)), nprocs=world, join=True)
    got = np.load(out)
    db, qs, keep = _data()
    want_d, want_i = oracle.topk(db, qs, k, metric, _words(keep))
    assert np.array_equal(got["i"], want_i)
    np.testing.assert_allclose(got["d"], want_d, rtol=1e-5)
