"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device and the built ``libmote_cuda.so``;
everything else runs on a CPU-only host.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import ref

    ref.build()
    return ref
