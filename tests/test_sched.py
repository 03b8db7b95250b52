"""CPU tests of the host runtime (include/gdn_host.h): the token scheduler, slot allocation,
slot-range sharding and step packing.  The first three mirror the reference's own scheduler
tests (src/scheduler/scheduler.rs:271-348) with the executor's work reduced to the plan
itself; the rest pin the packing tables and the slot life cycle."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.fixture(scope="module")
def sched(pkg):
    import importlib
    return importlib.import_module("qwen_mlx_b200.sched")


def _run(s, stop_fn=None, max_steps=1000):
    """Plan/complete until idle; returns the plans."""
    plans = []
    while s.has_work() and len(plans) < max_steps:
        p = s.plan()
        plans.append(p)
        s.complete([bool(stop_fn(e)) for e in p] if stop_fn else None)
    return plans


def test_single_sequence(sched):
    s = sched.TokenScheduler(max_batch=4)
    s.enqueue(prompt_len=3, max_tokens=5)
    assert s.pending_count() == 1
    p = s.plan()
    assert [(e.kind, e.n_tokens, e.pos) for e in p] == [(sched.PREFILL_FIRST, 3, 0)]
    s.complete()
    assert s.stats["active"] == 1
    plans = _run(s)
    # 1 token from the prompt, then 4 decode steps of one token
    assert [len(p) for p in plans] == [1, 1, 1, 1]
    assert [p[0].pos for p in plans] == [3, 4, 5, 6]
    assert not s.has_work()
    assert s.drain_finished() == [(1, sched.FINISH_MAX_TOKENS)]


def test_interleaved_sequences(sched):
    s = sched.TokenScheduler(max_batch=4)
    for t in ([1], [2], [3]):
        s.enqueue(len(t), 3)
    _run(s)
    st = s.stats
    assert st["total_requests"] == 3
    # each sequence: 1 prompt token + 2 decode tokens; only decode tokens are counted
    assert st["tokens_generated"] == 6
    assert st["free_slots"] == 256


def test_round_robin_fairness(sched):
    s = sched.TokenScheduler(max_batch=1)
    a = s.enqueue(1, 100)
    b = s.enqueue(1, 100)
    for _ in range(2):
        s.plan()
        s.complete()
    front = s.active_ids()
    assert sorted(front) == [a, b]
    p = s.plan()
    assert [e.seq_id for e in p] == [front[0]]
    s.complete()
    assert s.active_ids() == [front[1], front[0]]


def test_eos_stops_a_sequence_and_frees_its_slot(sched):
    s = sched.TokenScheduler(max_batch=8, slots_per_shard=4, prefill_budget=4)
    ids = [s.enqueue(2, 50) for _ in range(3)]
    s.plan()
    s.complete()
    assert s.free_slots(0) == 1
    p = s.plan()
    stop = [e.seq_id == ids[1] for e in p]
    s.complete(stop)
    assert s.drain_finished() == [(ids[1], sched.FINISH_EOS)]
    assert s.free_slots(0) == 2
    assert ids[1] not in s.active_ids()


def test_end_token_at_prompt_end_is_reported_as_eos(sched):
    s = sched.TokenScheduler(max_batch=2)
    sid = s.enqueue(4, 10)
    s.plan()
    s.complete([True])
    assert s.drain_finished() == [(sid, sched.FINISH_EOS)]
    # max_tokens == 1 also ends at the prompt, reported the same way as the reference's prefill path
    sid2 = s.enqueue(4, 1)
    s.plan()
    s.complete()
    assert s.drain_finished() == [(sid2, sched.FINISH_EOS)]


def test_full_pool_keeps_requests_waiting(sched):
    s = sched.TokenScheduler(max_batch=8, n_shards=2, slots_per_shard=2, prefill_budget=8)
    ids = [s.enqueue(1, 2) for _ in range(6)]
    p = s.plan()
    assert [e.seq_id for e in p] == ids[:4]
    # balanced over the shards, lowest free slot first within a shard
    assert sorted(e.slot for e in p) == [0, 1, 2, 3]
    assert [e.slot // 2 for e in p] == [0, 1, 0, 1]
    assert s.stats["waiting"] == 2
    s.complete()
    p = s.plan()          # 4 decode entries finish their 2 tokens; no slot is free yet
    assert all(e.kind == sched.DECODE for e in p) and len(p) == 4
    s.complete()
    assert s.stats["free_slots"] == 4
    p = s.plan()
    assert [e.seq_id for e in p] == ids[4:]


def test_chunked_prefill_positions_and_mixed_steps(sched):
    s = sched.TokenScheduler(max_batch=4, prefill_budget=1, prefill_chunk=4)
    a = s.enqueue(10, 3)
    b = s.enqueue(2, 3)
    plans = _run(s)
    rows = [[(e.seq_id, e.kind, e.n_tokens, e.pos) for e in p] for p in plans]
    F, C_, D = sched.PREFILL_FIRST, sched.PREFILL_CONT, sched.DECODE
    assert rows[0] == [(a, F, 4, 0)]
    assert rows[1] == [(a, C_, 4, 4), (b, F, 2, 0)]
    assert rows[2] == [(a, C_, 2, 8), (b, D, 1, 2)]
    # a's finished prompt joined the queue before b was requeued (prefills first, as the reference)
    assert rows[3] == [(a, D, 1, 10), (b, D, 1, 3)]
    assert rows[4] == [(a, D, 1, 11)]
    assert len(rows) == 5


def test_plan_complete_protocol_errors(sched, abi):
    s = sched.TokenScheduler(max_batch=2)
    with pytest.raises(abi.GdnError):
        s.complete()
    s.enqueue(1, 2)
    s.plan()
    with pytest.raises(abi.GdnError):
        s.plan()
    with pytest.raises(abi.GdnError):
        s.enqueue(0, 1)
    with pytest.raises(abi.GdnError):
        sched.TokenScheduler(max_batch=0)


def _pack_ref(entries, n_shards, per):
    """Plain restatement of gdn_pack_step's tables."""
    row0 = np.concatenate([[0], np.cumsum([e.n_tokens for e in entries])])
    out = []
    for s in range(n_shards):
        mine = [(i, e) for i, e in enumerate(entries) if e.slot // per == s]
        slots = [e.slot - s * per for _, e in mine]
        cu = np.concatenate([[0], np.cumsum([e.n_tokens for _, e in mine])]).astype(np.int32)
        rows = [r for i, e in mine for r in range(row0[i], row0[i] + e.n_tokens)]
        out.append((slots, cu.tolist(), rows))
    return out


def test_pack_step_tables_match_restatement(sched, synth):
    per, n_shards = 16, 4
    rng = np.random.default_rng(7)
    slots = rng.permutation(per * n_shards)[:23]
    entries = [sched.StepEntry(i + 1, int(sl), int(rng.integers(1, 9)), sched.DECODE, 0) for i, sl in enumerate(slots)]
    got = sched.pack_step(entries, n_shards, per)
    ref = _pack_ref(entries, n_shards, per)
    for t, (sl, cu, rows) in zip(got, ref):
        assert t.slot_ids.tolist() == sl
        assert t.cu_seqlens.tolist() == cu
        assert t.row_src.tolist() == rows
    # every row of the step lands on exactly one shard
    allrows = np.sort(np.concatenate([t.row_src for t in got]))
    assert allrows.tolist() == list(range(sum(e.n_tokens for e in entries)))


def test_pack_step_rejects_bad_entries(sched, abi):
    E = sched.StepEntry
    with pytest.raises(abi.GdnError):
        sched.pack_step([E(1, 3, 1, 0, 0), E(2, 3, 1, 0, 0)], 2, 4)   # slot twice
    with pytest.raises(abi.GdnError):
        sched.pack_step([E(1, 8, 1, 0, 0)], 2, 4)                     # outside the shards
    with pytest.raises(abi.GdnError):
        sched.pack_step([E(1, 2, 0, 0, 0)], 2, 4)                     # no rows
    empty = sched.pack_step([], 3, 4)
    assert [t.n_tokens for t in empty] == [0, 0, 0] and [t.cu_seqlens.tolist() for t in empty] == [[0], [0], [0]]


def test_scheduled_tables_pass_the_routing_validator(sched, abi):
    """Every shard table a scheduled workload produces is accepted by gdn_validate_tables."""
    import ctypes as C
    per, n_shards = 8, 2
    s = sched.TokenScheduler(max_batch=6, n_shards=n_shards, slots_per_shard=per, prefill_budget=3, prefill_chunk=16)
    rng = np.random.default_rng(3)
    for _ in range(30):
        s.enqueue(int(rng.integers(1, 60)), int(rng.integers(1, 12)))
    steps = 0
    while s.has_work():
        p = s.plan()
        for t in sched.pack_step(p, n_shards, per):
            rc = abi.lib().gdn_validate_tables(per, t.slot_ids.ctypes.data_as(C.c_void_p),
                                               t.cu_seqlens.ctypes.data_as(C.c_void_p), t.n_seq, t.n_tokens)
            assert rc == 0, abi.last_error()
        s.complete(rng.random(len(p)) < 0.05)
        steps += 1
    assert steps > 10 and s.stats["free_slots"] == per * n_shards
    assert len(s.drain_finished()) == 30


def test_shard_positions_track_the_kv_cache(sched):
    """positions[i] of a shard table is where sequence i's first token of the step goes in its slot's KV cache
    (the attention layers' gdn_attn_step): 0 after a PREFILL_FIRST reset, then the running token count."""
    per, n_shards = 8, 2
    s = sched.TokenScheduler(max_batch=6, n_shards=n_shards, slots_per_shard=per, prefill_budget=3, prefill_chunk=16)
    rng = np.random.default_rng(5)
    for _ in range(25):
        s.enqueue(int(rng.integers(1, 50)), int(rng.integers(1, 10)))
    kv_len = np.full((n_shards, per), -1)
    steps = 0
    while s.has_work():
        p = s.plan()
        for t in sched.pack_step(p, n_shards, per):
            for sl in t.reset_slots:
                kv_len[t.shard, sl] = 0
            lens = np.diff(t.cu_seqlens)
            assert t.positions.shape == t.slot_ids.shape
            for sl, pos, n in zip(t.slot_ids, t.positions, lens):
                assert kv_len[t.shard, sl] == pos
                kv_len[t.shard, sl] += n
        s.complete()
        steps += 1
    assert steps > 10
