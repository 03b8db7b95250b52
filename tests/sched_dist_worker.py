"""Worker of the sharded-scheduling test (tests/test_sched_dist.py), one process per rank.

Rank 0 runs the token scheduler and broadcasts each step's plan; every rank packs the
same per-shard tables, rank 0 routes the step's rows to the rank owning each shard and
gathers the outputs back (run_sharded_step).  The executor is a stand-in with a
per-slot state: for each token row x of a sequence, s <- 0.5 s + x and the output row is
s; a PREFILL_FIRST entry's slot starts from zero.  Its result depends only on the
sequence's own rows and on their order, so any routing mistake shows up.
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

HIDDEN = 8
WORKLOAD = dict(n_req=24, seed=11)


def requests():
    rng = np.random.default_rng(WORKLOAD["seed"])
    return [(int(rng.integers(1, 40)), int(rng.integers(1, 9))) for _ in range(WORKLOAD["n_req"])]


def token_row(seq_id: int, pos: int) -> np.ndarray:
    return np.sin(0.37 * seq_id + 0.11 * pos + 0.05 * np.arange(HIDDEN)).astype(np.float32)


def stops(entry) -> bool:
    """A deterministic end token: sequence 5 ends at its first decode, sequence 9 at its prompt."""
    return (entry.seq_id == 5 and entry.kind == 0) or (entry.seq_id == 9 and entry.kind != 0)


class MockShard:
    def __init__(self, n_slots):
        self.state = np.zeros((n_slots, HIDDEN), np.float64)
        self.slots_seen = set()

    def run(self, tables, x):
        import torch
        xs = x.double().numpy()
        y = np.empty_like(xs)
        for s in tables.reset_slots:
            self.state[s] = 0.0
        for i in range(tables.n_seq):
            sl = int(tables.slot_ids[i])
            self.slots_seen.add(sl)
            for r in range(int(tables.cu_seqlens[i]), int(tables.cu_seqlens[i + 1])):
                self.state[sl] = 0.5 * self.state[sl] + xs[r]
                y[r] = self.state[sl]
        return torch.from_numpy(y.astype(np.float32))


def drive(n_shards, per, rank, world, dist):
    """Run the workload; rank 0 returns {(seq_id, position): output row}."""
    import torch
    import __graft_entry__ as ge
    ge.load_package()
    from qwen_mlx_b200 import sched
    shard = MockShard(per)
    s = sched.TokenScheduler(max_batch=5, n_shards=n_shards, slots_per_shard=per, prefill_budget=2,
                             prefill_chunk=16) if rank == 0 else None
    if rank == 0:
        for p, m in requests():
            s.enqueue(p, m)
    outputs = {}
    steps = 0
    while True:
        plan = [s.plan() if s.has_work() else None] if rank == 0 else [None]
        if dist is not None:
            dist.broadcast_object_list(plan, src=0)
        entries = plan[0]
        if entries is None:
            break
        tables = sched.pack_step(entries, n_shards, per)
        rows = None
        if rank == 0:
            rows = torch.from_numpy(np.concatenate(
                [np.stack([token_row(e.seq_id, e.pos + t) for t in range(e.n_tokens)]) for e in entries]))
        if dist is None:
            for t in tables:
                if t.n_tokens:
                    rows[torch.from_numpy(t.row_src).long()] = shard.run(t, rows[torch.from_numpy(t.row_src).long()])
        else:
            sched.run_sharded_step(entries, tables, rows, shard.run, dist, rank, world)
        if rank == 0:
            r = 0
            for e in entries:
                for t in range(e.n_tokens):
                    outputs[(e.seq_id, e.pos + t)] = rows[r].numpy().copy()
                    r += 1
            s.complete([stops(e) for e in entries])
        steps += 1
    return outputs, sorted(shard.slots_seen), steps


def main(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        outputs, seen, steps = drive(world, 6, rank, world, dist)
        np.save(Path(out_dir) / f"rank{rank}.npy", np.array([outputs, seen, steps], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4])
