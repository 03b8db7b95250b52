"""Slot-range sharding over two ranks (gloo on CPU, world_size 2).

Two processes run tests/sched_dist_worker.py: rank 0 schedules a mixed prefill/decode
workload over 2 shards x 6 slots and routes each step's rows to the rank owning each
shard; each rank runs a stand-in executor over its own slots.  The per-token outputs
must equal, bit for bit, a single-process run of the same workload on one 12-slot shard,
and each rank must have touched only its own slot range."""
from __future__ import annotations

import socket
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import sched_dist_worker as W  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_sharded_schedule_matches_single_process(tmp_path, pkg):
    ref, seen1, steps1 = W.drive(1, 12, 0, 1, None)
    port = _free_port()
    procs = [subprocess.Popen([sys.executable, str(HERE / "sched_dist_worker.py"), str(r), "2", str(port),
                               str(tmp_path)], stdout=subprocess.PIPE, stderr=subprocess.STDOUT) for r in range(2)]
    logs = []
    try:
        for p in procs:
            out, _ = p.communicate(timeout=240)
            logs.append(out.decode(errors="replace"))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)
    r0 = np.load(tmp_path / "rank0.npy", allow_pickle=True)
    r1 = np.load(tmp_path / "rank1.npy", allow_pickle=True)
    outputs, seen0, steps = r0
    _, seen_1, steps_r1 = r1
    assert steps == steps1 == steps_r1
    assert set(outputs) == set(ref)
    for key, row in ref.items():
        assert np.array_equal(outputs[key], row), key
    # both shards worked, each only on its local slots 0..5
    assert seen0 and seen_1
    assert max(seen0) < 6 and max(seen_1) < 6
    # the workload finished with every prompt token and decode token accounted for
    n_rows = sum(p + m - 1 for p, m in W.requests())
    assert len(ref) <= n_rows
