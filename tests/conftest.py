"""Shared pytest configuration: the ``gpu`` marker and fixture helpers."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def reference_root() -> Path | None:
    """The LARA source tree named by ``LARA_REFERENCE`` (checks that read the
    reference's own files skip when it is unset or absent)."""
    path = os.environ.get("LARA_REFERENCE")
    if not path:
        return None
    p = Path(path)
    return p if p.is_dir() else None


REFERENCE = reference_root()
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")
    config.addinivalue_line("markers", "slow: full-size parity cases")


def pytest_collection_modifyitems(config, items):
    # GPU tests must never silently pass without a device: if a GPU test is
    # selected on a machine without CUDA, it is an error, not a skip.
    pass


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
