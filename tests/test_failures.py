"""Failure handling, with no GPU fault (nothing traps, faults or hangs).

GPU:
- a bounded pipeline wait of the tcgen05 search runs out on purpose (the
  producer loads nothing and every wait gets a short poll limit, both
  test-only switches): the call returns, cr_filtered_topk_check reports
  CR_ERR_DEVICE, and the next search on the same context is correct;
- device allocations fail by injection (cr_test_fail_allocations) inside
  uploads, set operations and the search: each call raises CR_ERR_OOM
  (-3) cleanly and the same calls succeed, with correct results, once the
  injection is off.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(n, q, seed=0):
    rng = np.random.default_rng(seed)
    db = rng.standard_normal((n, 128)).astype(np.float32)
    db /= np.linalg.norm(db, axis=1, keepdims=True)
    qs = rng.standard_normal((q, 128)).astype(np.float32)
    qs /= np.linalg.norm(qs, axis=1, keepdims=True)
    return db.astype(np.float16), qs.astype(np.float16)


def test_pipeline_wait_runs_out_and_is_reported(cr, oracle, monkeypatch):
    import torch

    from checks import check_topk

    db, qs = _data(20_000, 33)
    ddb, dq = torch.from_numpy(db).cuda(), torch.from_numpy(qs).cuda()
    monkeypatch.setenv("CR_TOPK_DEBUG", "7")
    monkeypatch.setenv("CR_TOPK_SPIN_LIMIT", "4096")
    cr.filtered_topk(ddb, dq, 10)
    rc = cr.lib().cr_filtered_topk_check()
    assert rc == -5, f"expected CR_ERR_DEVICE, got {rc}"
    assert "timed out" in cr.lib().cr_last_error_string().decode()
    monkeypatch.delenv("CR_TOPK_DEBUG")
    monkeypatch.delenv("CR_TOPK_SPIN_LIMIT")
    d, i = cr.filtered_topk(ddb, dq, 10)
    assert cr.lib().cr_filtered_topk_check() == 0
    d_ref, i_ref = oracle.topk(db, qs, 10, 0, None)
    check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, "after the failed wait")


@pytest.mark.parametrize("after", [0, 1, 2])
def test_injected_allocation_failures(cr, oracle, after):
    import torch

    rng = np.random.default_rng(after)
    u = 1 << 20
    a_ids = rng.integers(0, u, 40_000, dtype=np.uint64).astype(np.uint32)
    b_ids = np.flatnonzero(rng.random(u) < 0.7).astype(np.uint32)
    a = cr.upload_from_ids(a_ids, u)
    b = cr.upload_from_ids(b_ids, u)
    db, qs = _data(8192, 16, seed=after)
    ddb, dq = torch.from_numpy(db).cuda(), torch.from_numpy(qs).cuda()
    calls = [lambda: cr.upload_from_ids(a_ids, u), lambda: cr.set_operation(a, b, cr.ANDNOT),
             lambda: cr.multi_and([a, b, a]), lambda: cr.upload_from_device_bitset(cr.decompress_to_bitset(b), u)]
    try:
        for fn in calls:
            cr.lib().cr_test_fail_allocations(after)
            try:
                r = fn()
            except RuntimeError as e:
                assert "(-3)" in str(e), str(e)
            else:
                r.free()  # enough allocations were left for this call
        cr.lib().cr_test_fail_allocations(0)
        with pytest.raises(RuntimeError, match=r"\(-3\)"):
            cr.upload_from_ids(a_ids, u)
    finally:
        cr.lib().cr_test_fail_allocations(-1)
    torch.cuda.synchronize()
    r = cr.set_operation(a, b, cr.ANDNOT)
    want = oracle.set_operation(oracle.from_ids(a_ids, u), oracle.from_ids(b_ids, u), cr.ANDNOT).enumerate()
    assert np.array_equal(cr.enumerate_ids(r, dtype="uint32").cpu().numpy().view(np.uint32), want)
    d, i = cr.filtered_topk(ddb, dq, 5)
    d_ref, i_ref = oracle.topk(db, qs, 5, 0, None)
    from checks import check_topk

    check_topk(d.cpu().numpy(), i.cpu().numpy(), d_ref, i_ref, "after injection")
    for x in (a, b, r):
        x.free()
