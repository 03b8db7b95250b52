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


# The reference fixes no accumulation order for its projection GEMMs (MLX matmul).  Parity
# cases that include projections run the oracle with its default (sequential) order and with
# three other valid orders; the spread between them calibrates the tolerance.
ALT_ORDERS = (1, 2, 3)


def with_order(oracle, order, fn):
    oracle.set_linear_order(order)
    try:
        return fn()
    finally:
        oracle.set_linear_order(0)


def order_noise(ref, alts, conv=lambda a: a):
    """Largest distance between the default-order oracle and the other-order runs."""
    return max(rel_l2(conv(a), conv(ref)) for a in alts)
