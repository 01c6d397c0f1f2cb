"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device and the built ``librwkv_b200.so``;
everything else runs on CPU (oracle vs golden vectors, host logic, the C-ABI
library's exported symbols, multi-rank sharding over ``gloo``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built CUDA library")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
