"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device with the compiled ``serron_b200`` library;
everything else runs on a CPU-only machine.
"""

from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the compiled serron_b200 library")
    config.addinivalue_line("markers", "slow: long-running")
