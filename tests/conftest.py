"""Shared pytest setup: import paths, the `gpu` marker, fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_DIR = REPO / "cu-roaring-bitmap_b200"
for p in (REPO, PKG_DIR, REPO / "oracle", REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def built_lib():
    """Builds (if stale) and returns the path of libcuroaring_b200.so."""
    import build

    return build.build_lib()


@pytest.fixture(scope="session")
def cr(built_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import cu_roaring_b200

    return cu_roaring_b200
