"""CPU checks of the workload definitions in bench.py: the config-5 step plans (sharded serving) are what the
workload states — every one of a GPU's 256 slots steps each time, 10% of them with a prefill chunk of U[64, 1024]
tokens and the rest one decode token, packed in a random order, seeded per rank."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config5_plans_follow_the_workload(bench):
    plans, ctx = bench.config5_plans(rank=0, n_steps=6)
    assert len(plans) == 6
    assert ctx.shape == (256,) and ctx.min() >= 16 and ctx.max() <= 32768
    for slots, cu in plans:
        assert sorted(slots.tolist()) == list(range(256))          # every slot steps once
        lens = np.diff(cu)
        assert cu[0] == 0 and len(lens) == 256
        chunks = lens[lens > 1]
        assert len(chunks) == 26                                    # round(10% of 256)
        assert chunks.min() >= 64 and chunks.max() <= 1024
        assert np.all(lens[lens <= 1] == 1)
    # the chunks are not all packed first
    assert any(np.argmax(np.diff(cu) > 1) > 0 for _, cu in plans)


def test_config5_plans_differ_by_rank_and_repeat_by_seed(bench):
    a, _ = bench.config5_plans(rank=0, n_steps=3)
    b, _ = bench.config5_plans(rank=1, n_steps=3)
    a2, _ = bench.config5_plans(rank=0, n_steps=3)
    assert any(not np.array_equal(x[1], y[1]) for x, y in zip(a, b))
    assert all(np.array_equal(x[0], y[0]) and np.array_equal(x[1], y[1]) for x, y in zip(a, a2))
