"""Shared test configuration.

Markers: `gpu` tests need a CUDA device (run on a B200 with `-m gpu`); all
other tests run on the CPU. The reference build (oracle/_ref) and the CPU
oracle library are test infrastructure built by `__graft_entry__.build()`.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
REF_LIBRARY = REPO / "oracle" / "_ref" / "libref_hybridsplat.so"
REF_PREPARE = REPO / "oracle" / "_ref" / "libref_prepare.so"
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """Loader for tests/golden/<name>.npz (skips when fixtures are absent)."""

    def load(name: str) -> dict:
        path = GOLDEN / f"{name}.npz"
        if not path.exists():
            pytest.skip(f"golden fixture {path.name} not generated")
        with np.load(path) as data:
            return {k: data[k] for k in data.files}

    return load


@pytest.fixture(scope="session")
def ref_library():
    """The reference library rebuilt for Blackwell (oracle/_ref), if present."""
    if not REF_LIBRARY.exists():
        pytest.skip("reference build oracle/_ref/libref_hybridsplat.so is absent")
    from hybridsplat_jittor_render_b200.native_runtime import bind_library

    return bind_library(REF_LIBRARY, require_optix=False)
