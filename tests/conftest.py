"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as ge  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return ge.load_package()


@pytest.fixture(scope="session")
def synth(pkg):
    import importlib
    return importlib.import_module("qwen_mlx_b200.synth")


@pytest.fixture(scope="session")
def oracle():
    return ge.load_oracle()


@pytest.fixture(scope="session")
def gdn(pkg):
    import importlib
    return importlib.import_module("qwen_mlx_b200.gdn")


@pytest.fixture(scope="session")
def abi(pkg):
    import importlib
    return importlib.import_module("qwen_mlx_b200.abi")


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))
