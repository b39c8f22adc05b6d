"""GPU: the fused filtered top-k (tcgen05 GEMM + bitmap predicate + select)
against the exact fp32 oracle.

Tolerance: distances within 1e-3 relative; id sets
equal except where the oracle's k-th distance ties within that tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def make_data(n, q, dim=128, seed=0):
    rng = np.random.default_rng(seed)
    db = rng.standard_normal((n, dim)).astype(np.float32)
    db /= np.linalg.norm(db, axis=1, keepdims=True)
    qs = rng.standard_normal((q, dim)).astype(np.float32)
    qs /= np.linalg.norm(qs, axis=1, keepdims=True)
    return db.astype(np.float16), qs.astype(np.float16)


def check_topk(d_gpu, i_gpu, d_ref, i_ref, metric):
    from checks import check_topk as _check

    _check(d_gpu, i_gpu, d_ref, i_ref, f"metric {metric}")


@pytest.fixture(scope="module")
def torch_():
    import torch

    return torch


@pytest.mark.parametrize("n,q,k", [(5000, 37, 10), (20000, 300, 100), (70001, 129, 256), (1000, 5, 1)])
@pytest.mark.parametrize("metric", [0, 1])
@pytest.mark.parametrize("pass_rate", [None, 0.5, 0.01])
def test_topk_matches_oracle(cr, oracle, torch_, n, q, k, metric, pass_rate):
    db, qs = make_data(n, q, seed=n + q)
    filt = None
    pass_bits = None
    if pass_rate is not None:
        rng = np.random.default_rng(3)
        ids = np.flatnonzero(rng.random(n) < pass_rate).astype(np.uint32)
        filt = cr.upload_from_ids(ids, n)
        words = np.zeros((n + 31) // 32, dtype=np.uint32)
        np.bitwise_or.at(words, ids // 32, (1 << (ids % 32)).astype(np.uint32))
        pass_bits = words
    d_ref, i_ref = oracle.topk(db, qs, k, metric, pass_bits)
    ddb = torch_.from_numpy(db).cuda()
    dq = torch_.from_numpy(qs).cuda()
    norms = cr.row_norms(ddb) if metric == 1 else None
    d, i = cr.filtered_topk(ddb, dq, k, metric=metric, filter=filt, db_norms=norms)
    check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, metric)
    if filt is not None:
        filt.free()


def test_topk_row_offset_and_merge(cr, oracle, torch_):
    """Sharded search: two row ranges with global IDs, then cr_topk_merge."""
    n, q, k = 30000, 64, 50
    db, qs = make_data(n, q, seed=9)
    rng = np.random.default_rng(4)
    ids = np.flatnonzero(rng.random(n) < 0.1).astype(np.uint32)
    filt = cr.upload_from_ids(ids, n)
    words = np.zeros((n + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(words, ids // 32, (1 << (ids % 32)).astype(np.uint32))
    for metric in (0, 1):
        d_ref, i_ref = oracle.topk(db, qs, k, metric, words)
        dq = torch_.from_numpy(qs).cuda()
        parts_d, parts_i = [], []
        for lo, hi in ((0, 12288), (12288, n)):
            ddb = torch_.from_numpy(np.ascontiguousarray(db[lo:hi])).cuda()
            d, i = cr.filtered_topk(ddb, dq, k, metric=metric, filter=filt, row_offset=lo)
            parts_d.append(d)
            parts_i.append(i)
        d, i = cr.topk_merge(torch_.stack(parts_d), torch_.stack(parts_i), k, metric=metric)
        check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, metric)
    filt.free()


def test_topk_against_torch_fp32_large(cr, torch_):
    """1M x 128, 1000 queries, k=100, 10% pass: against torch fp32 matmul."""
    n, q, k = 1_000_000, 1000, 100
    g = torch_.Generator(device="cuda").manual_seed(5)
    db = torch_.nn.functional.normalize(torch_.randn(n, 128, device="cuda", generator=g), dim=1).half()
    qs = torch_.nn.functional.normalize(torch_.randn(q, 128, device="cuda", generator=g), dim=1).half()
    keep = torch_.rand(n, device="cuda", generator=g) < 0.1
    ids = torch_.nonzero(keep).flatten().to(torch_.int32)
    filt = cr.upload_from_ids(ids, n)
    d, i = cr.filtered_topk(db, qs, k, metric=0, filter=filt)
    scores = qs.float() @ db.float().T
    scores[:, ~keep] = -float("inf")
    ref_d, ref_i = torch_.topk(scores, k, dim=1)
    check_topk(d.cpu().numpy(), i.cpu().numpy(), ref_d.cpu().numpy(), ref_i.cpu().numpy(), 0)
    filt.free()


def test_topk_no_passing_rows(cr, torch_):
    """A filter that excludes every row of the shard: every slot is (inf/-inf, -1)."""
    db, qs = make_data(4096, 20, seed=2)
    filt = cr.upload_from_ids(np.array([5000, 6000], np.uint32), 10000)  # rows outside [0, 4096)
    for metric in (0, 1):
        d, i = cr.filtered_topk(torch_.from_numpy(db).cuda(), torch_.from_numpy(qs).cuda(), 7, metric=metric,
                                filter=filt)
        assert (i.cpu().numpy() == -1).all()
        assert np.isinf(d.cpu().numpy()).all()
    filt.free()


def test_topk_all_ties_falls_back_exactly(cr, torch_):
    """Every row identical: all scores tie, the candidate arrays overflow and
    the search redoes the batch with per-list merging; ties go to the
    smallest ids."""
    n, q, k = 200_000, 40, 10
    row = np.random.default_rng(0).standard_normal(128).astype(np.float32)
    row /= np.linalg.norm(row)
    db = np.tile(row.astype(np.float16), (n, 1))
    _, qs = make_data(10, q, seed=4)
    for metric in (0, 1):
        d, i = cr.filtered_topk(torch_.from_numpy(db).cuda(), torch_.from_numpy(qs).cuda(), k, metric=metric)
        assert (i.cpu().numpy() == np.arange(k)[None, :]).all()


@pytest.mark.parametrize("kind", ["runs", "runs_dense", "negated", "array_sparse", "offset_not_32"])
def test_topk_filter_container_kinds(cr, oracle, torch_, kind):
    """Filters made of RUN containers, a negated (complement-stored) filter,
    sparse ARRAY containers, and a shard offset that is not a multiple of 32
    (per-row membership path)."""
    n, q, k = 140_000, 50, 20
    db, qs = make_data(n, q, seed=11)
    rng = np.random.default_rng(8)
    if kind == "runs":
        ids = np.concatenate([np.arange(s, s + 3000) for s in range(0, n - 3000, 9000)]).astype(np.uint32)
    elif kind == "runs_dense":  # ~80% pass in long runs: searched densely, mostly full mask words
        ids = np.concatenate([np.arange(s, min(n, s + 8000)) for s in range(0, n, 10000)]).astype(np.uint32)
    elif kind == "negated":
        ids = np.flatnonzero(rng.random(n) < 0.9).astype(np.uint32)
    else:
        ids = np.flatnonzero(rng.random(n) < 0.003).astype(np.uint32)
    lo = 0 if kind != "offset_not_32" else 1000 + 7
    filt = cr.upload_from_ids(ids, n, bitmap_threshold=4096)
    if kind in ("runs", "runs_dense"):
        assert filt.raw.n_run_containers > 0 or filt.raw.negated
    if kind == "negated":
        assert filt.raw.negated
    words = np.zeros((n + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(words, ids // 32, (1 << (ids % 32)).astype(np.uint32))
    shard = db[lo:]
    sub = np.zeros(((n - lo) + 31) // 32, dtype=np.uint32)
    sel = ids[ids >= lo] - lo
    np.bitwise_or.at(sub, sel // 32, (1 << (sel % 32)).astype(np.uint32))
    d_ref, i_ref = oracle.topk(shard, qs, k, 0, sub)
    i_ref = np.where(i_ref >= 0, i_ref + lo, -1)
    d, i = cr.filtered_topk(torch_.from_numpy(np.ascontiguousarray(shard)).cuda(), torch_.from_numpy(qs).cuda(),
                            k, metric=0, filter=filt, row_offset=lo)
    check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, 0)
    filt.free()


@pytest.mark.parametrize("n_dup", [60, 600])
def test_topk_duplicate_rows_tie_break(cr, oracle, torch_, n_dup):
    """n_dup copies of query 0's own vector planted among random rows: for
    query 0 they tie for first place and the smallest ids of them must come
    out, in id order. 600 copies exceed the exact-rank pass of the merge and
    take its sorting fallback; 60 copies stay on the rank pass."""
    n, q, k = 60_000, 64, 100
    db, qs = make_data(n, q, seed=21)
    rng = np.random.default_rng(22)
    dup = np.sort(rng.choice(n, n_dup, replace=False))
    db[dup] = qs[0]
    ids = np.flatnonzero(rng.random(n) < 0.3).astype(np.uint32)
    ids = np.union1d(ids, dup).astype(np.uint32)
    filt = cr.upload_from_ids(ids, n)
    words = np.zeros((n + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(words, ids // 32, (1 << (ids % 32)).astype(np.uint32))
    for metric in (0, 1):
        d_ref, i_ref = oracle.topk(db, qs, k, metric, words)
        ddb = torch_.from_numpy(db).cuda()
        d, i = cr.filtered_topk(ddb, torch_.from_numpy(qs).cuda(), k, metric=metric, filter=filt)
        i = i.cpu().numpy()
        m = min(k, n_dup)
        assert (i[0, :m] == dup[:m]).all()
        check_topk(d.cpu().numpy(), i, d_ref, i_ref, metric)
    filt.free()


@pytest.mark.parametrize("spec_j", ["1", "0"])
def test_topk_speculative_bound_verified(cr, oracle, torch_, monkeypatch, spec_j):
    """The speculative bound forced to the prologue sample's single best score
    (above the k-th best for nearly every query): the merge must detect it and
    the batch be redone without it. And with the bound switched off."""
    monkeypatch.setenv("CR_TOPK_SPEC_J", spec_j)
    n, q, k = 400_000, 200, 50
    db, qs = make_data(n, q, seed=31)
    rng = np.random.default_rng(32)
    ids = np.flatnonzero(rng.random(n) < 0.2).astype(np.uint32)
    filt = cr.upload_from_ids(ids, n)
    words = np.zeros((n + 31) // 32, dtype=np.uint32)
    np.bitwise_or.at(words, ids // 32, (1 << (ids % 32)).astype(np.uint32))
    for metric in (0, 1):
        d_ref, i_ref = oracle.topk(db, qs, k, metric, words)
        d, i = cr.filtered_topk(torch_.from_numpy(db).cuda(), torch_.from_numpy(qs).cuda(), k, metric=metric,
                                filter=filt)
        check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, metric)
    filt.free()


def test_topk_merge_packed(cr, oracle, torch_):
    """Two shards' results written into packed blocks (distances then ids, as
    one collective would carry them) and merged in place."""
    n, q, k = 30000, 64, 50
    db, qs = make_data(n, q, seed=19)
    dq = torch_.from_numpy(qs).cuda()
    for metric in (0, 1):
        d_ref, i_ref = oracle.topk(db, qs, k, metric, None)
        blocks = []
        for lo, hi in ((0, 17000), (17000, n)):
            block, bd, bi = cr.topk_packed_buffer(q, k, "cuda")
            ddb = torch_.from_numpy(np.ascontiguousarray(db[lo:hi])).cuda()
            cr.filtered_topk(ddb, dq, k, metric=metric, row_offset=lo, out_dist=bd, out_ids=bi)
            blocks.append(block)
        d, i = cr.topk_merge_packed(torch_.stack(blocks), q, k, metric=metric)
        check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, metric)
