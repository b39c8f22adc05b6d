"""CPU: the oracle's multi_and / multi_or over more than 64 inputs (chained
passes of 64, then 63 plus the running result) equal the plain set algebra."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.mark.parametrize("count", [64, 65, 127, 200])
@pytest.mark.parametrize("fn", ["and", "or"])
def test_chained_multi_is_set_algebra(oracle, count, fn):
    u = 1 << 17
    rng = np.random.default_rng(count + (fn == "or"))
    words = []
    for i in range(count):
        p = 0.03 if i % 9 == 4 else 0.993
        m = rng.random(u) < p
        w = np.packbits(m, bitorder="little").view(np.uint32)
        words.append(w)
    ims = [oracle.from_bitset(w, u) for w in words]
    r = (oracle.multi_and if fn == "and" else oracle.multi_or)(ims)
    assert r.validate() == 0
    want = words[0].copy()
    for w in words[1:]:
        want = (want & w) if fn == "and" else (want | w)
    assert np.array_equal(r.decompress(), want)
