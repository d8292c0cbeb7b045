"""Shared pytest configuration.

Markers: ``gpu`` -- needs a CUDA device (B200) and the built ``libccut_moe.so``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
