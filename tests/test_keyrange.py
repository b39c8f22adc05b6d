"""Key-range sharding (cr_key_range / cr_key_slice / cr_concat_key_slices):
G ranks each hold one contiguous range of container keys of every operand,
compute with no communication, and the result slices laid end to end are
the unsharded result, container for container.

GPU: slices of engine bitmaps through set_operation, multi_and / multi_or and
contains, concatenated, bit-exact against the unsharded engine result and
the CPU oracle. CPU (two gloo ranks): the split itself, restated with the
oracle on logical sets, covers every ID once."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from checks import assert_same_image

AND, OR, ANDNOT, XOR = 0, 1, 2, 3


def _sets(u, seed):
    """Mixed containers: sparse uniform (ARRAY), dense Bernoulli (BITMAP, one
    operand complement-stored), runs (RUN)."""
    rng = np.random.default_rng(seed)
    a = rng.integers(0, u, u // 40, dtype=np.uint64).astype(np.uint32)
    b = np.flatnonzero(rng.random(u) < 0.6).astype(np.uint32)
    starts = np.arange(0, u - 3000, 7000)
    c = np.concatenate([np.arange(s, s + 2500) for s in starts]).astype(np.uint32)
    d = np.flatnonzero(rng.random(u) < 0.3).astype(np.uint32)
    return [a, b, c, d]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3, 5])
def test_sharded_set_ops_equal_unsharded(cr, oracle, world):
    import torch

    u = (37 << 16) + 1234  # a partial last chunk
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    ids = _sets(u, world)
    full = [cr.upload_from_ids(x, u) for x in ids]
    ora = [oracle.from_ids(x, u, 0xFFFFFFFF, l2) for x in ids]
    assert full[1].raw.negated
    ranges = [cr.key_range(u, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == (u + 65535) >> 16
    assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
    slices = [[cr.key_slice(b, lo, hi) for b in full] for lo, hi in ranges]
    # Slices of one operand put back together are the operand itself.
    for j, b in enumerate(full):
        cat = cr.concat_key_slices([slices[r][j] for r in range(world)])
        assert_same_image(cat.image(), b.image(), f"operand {j}")
        cat.free()
    cases = [("and", lambda x: cr.set_operation(x[0], x[3], AND), lambda o: oracle.set_operation(o[0], o[3], AND)),
             ("or", lambda x: cr.set_operation(x[1], x[2], OR), lambda o: oracle.set_operation(o[1], o[2], OR)),
             ("andnot", lambda x: cr.set_operation(x[3], x[1], ANDNOT),
              lambda o: oracle.set_operation(o[3], o[1], ANDNOT)),
             ("xor", lambda x: cr.set_operation(x[2], x[3], XOR), lambda o: oracle.set_operation(o[2], o[3], XOR)),
             ("multi_and", lambda x: cr.multi_and([x[1], x[3], x[0]]), lambda o: oracle.multi_and([o[1], o[3], o[0]])),
             ("multi_or", lambda x: cr.multi_or([x[0], x[1], x[2]]), lambda o: oracle.multi_or([o[0], o[1], o[2]]))]
    for name, fn, ofn in cases:
        parts = [fn(slices[r]) for r in range(world)]
        cat = cr.concat_key_slices(parts)
        whole = fn(full)
        assert_same_image(cat.image(), whole.image(), f"{name}: concatenated vs unsharded")
        assert_same_image(cat.image(), ofn(ora).image(), f"{name}: concatenated vs oracle")
        for p in parts + [cat, whole]:
            p.free()
    # Point queries: each rank answers the candidates of its key range.
    rng = np.random.default_rng(1)
    q = rng.integers(0, u, 200_000, dtype=np.uint64).astype(np.uint32)
    want = ora[1].contains(q)
    got = np.zeros(q.size, dtype=bool)
    for r, (lo, hi) in enumerate(ranges):
        sel = np.flatnonzero(((q >> 16) >= lo) & ((q >> 16) < hi))
        if sel.size == 0:
            continue
        bits = cr.contains_batch(slices[r][1], torch.from_numpy(q[sel].view(np.int32)).cuda())
        got[sel] = np.unpackbits(bits.cpu().numpy().view(np.uint8), bitorder="little")[:sel.size].astype(bool)
    assert np.array_equal(np.packbits(got, bitorder="little").view(np.uint32)[:want.size], want)
    for row in slices:
        for b in row:
            b.free()
    for b in full:
        b.free()


@pytest.mark.gpu
def test_slice_edges(cr):
    u = 5 << 16
    b = cr.upload_from_ids(np.array([1, 70000, 200000, 300000], np.uint32), u)
    e = cr.key_slice(b, 2, 2)
    assert e.raw.n_containers == 0 and e.raw.total_cardinality == 0 and e.raw.universe_size == u
    one = cr.key_slice(b, 1, 2)
    assert one.raw.n_containers == 1 and one.raw.total_cardinality == 1
    assert cr.enumerate_ids(one, dtype="uint32").cpu().numpy().view(np.uint32).tolist() == [70000]
    with pytest.raises(RuntimeError):
        cr.concat_key_slices([one, cr.key_slice(b, 0, 2)])  # overlapping / descending keys
    for x in (b, e, one):
        x.free()


# ----------------------------------------------------------- CPU, gloo

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, out_path):
    import torch.distributed as dist

    import cu_roaring_b200 as cr
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    u = (23 << 16) + 77
    ids = _sets(u, 9)
    lo, hi = cr.key_range(u, rank, world)
    mine = [x[((x >> 16) >= lo) & ((x >> 16) < hi)] for x in ids]  # this rank's IDs of each operand
    ims = [oracle.from_ids(x, u) for x in mine]
    part = oracle.multi_and([ims[1], ims[3]]).enumerate()
    allp = [None] * world if rank == 0 else None
    dist.gather_object(part, allp, dst=0)
    if rank == 0:
        np.save(out_path, np.concatenate(allp))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_key_split_covers_every_id_gloo(tmp_path, oracle, world):
    """Two gloo ranks bucket each operand's IDs by cr_key_range, AND their
    buckets (oracle), and rank 0 lays the parts end to end: the unsharded AND."""
    import torch.multiprocessing as mp

    out = tmp_path / "cat.npy"
    mp.start_processes(_gloo_rank, args=(world, _free_port(), str(out)), nprocs=world, join=True,
                       start_method="spawn")
    u = (23 << 16) + 77
    ids = _sets(u, 9)
    want = oracle.multi_and([oracle.from_ids(ids[1], u), oracle.from_ids(ids[3], u)]).enumerate()
    assert np.array_equal(np.load(out), want)
