"""Test configuration: import paths and the `gpu` marker.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on CPU.
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tt-infinity_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(params=["one_wave", "persistent"])
def copy_engine(request):
    """Runs a GPU test twice: with every copy whose grid allows it on the one-wave engine, and with
    every copy on the persistent engines (bulk or LDG), so each engine is checked on the same cases."""
    from kvcache_manager import _native

    lib = _native.load()
    assert lib.kvs_set_small_copy_limit(1 << 62 if request.param == "one_wave" else 0) == 0
    yield request.param
    assert lib.kvs_set_small_copy_limit(-1) == 0
