"""Host runtime around the GDN step, for Python callers.

* ``TokenScheduler`` binds the C++ token scheduler of include/gdn_host.h: the continuous
  batching policy of TokenScheduler (src/scheduler/scheduler.rs:36-174) with slots of a
  device pool as the per-sequence state and slot-range sharding over GPUs.  ``plan()``
  returns one step as a list of entries (prefill chunks first, then decode tokens) that
  runs as ONE packed ragged call per GPU; ``complete(stop)`` feeds back which entries
  produced an end token.
* ``pack_step`` splits a step into per-shard tables (local slot ids, cu_seqlens, and the
  rows of the step's packed input each shard takes).
* ``StackExecutor`` is the ModelExecutor side (src/scheduler/executor.rs:21-49) for the GDN
  stack on one GPU: it resets the slots of newly admitted sequences, then runs the 30-layer
  residual stack over the shard's rows in one ``gdn_stack_step`` call.  ``submit``/``collect``
  are the stream-ordered launch and the event wait of submit_batch / collect_batch.
* ``run_sharded_step`` moves a planned step's rows between rank 0 (which plans) and the
  rank owning each shard with torch.distributed point-to-point calls (host plumbing; the
  GDN step itself exchanges nothing between GPUs).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import abi

DECODE = abi.GDN_ENTRY_DECODE
PREFILL_FIRST = abi.GDN_ENTRY_PREFILL_FIRST
PREFILL_CONT = abi.GDN_ENTRY_PREFILL_CONT
FINISH_EOS = abi.GDN_FINISH_EOS
FINISH_MAX_TOKENS = abi.GDN_FINISH_MAX_TOKENS


@dataclass(frozen=True)
class StepEntry:
    seq_id: int
    slot: int       # global slot
    n_tokens: int
    kind: int       # DECODE / PREFILL_FIRST / PREFILL_CONT
    pos: int        # tokens of the sequence processed before this step


@dataclass
class ShardTables:
    shard: int
    slot_ids: np.ndarray    # int32 [n_seq] local slots
    cu_seqlens: np.ndarray  # int32 [n_seq + 1]
    row_src: np.ndarray     # int32 [n_tokens] row of the step's packed input
    reset_slots: np.ndarray  # int32 local slots to reset before the step (PREFILL_FIRST entries)
    positions: np.ndarray = None  # int32 [n_seq] tokens each sequence processed before this step: the KV-cache
                                  # position of its first token here (gdn_attn_step's `positions`)

    @property
    def n_seq(self) -> int:
        return int(self.slot_ids.shape[0])

    @property
    def n_tokens(self) -> int:
        return int(self.row_src.shape[0])


def _entries_c(entries):
    arr = (abi.GdnStepEntryC * max(len(entries), 1))()
    for i, e in enumerate(entries):
        arr[i] = abi.GdnStepEntryC(e.seq_id, e.slot, e.n_tokens, e.kind, e.pos)
    return arr


def pack_step(entries, n_shards: int, slots_per_shard: int) -> list[ShardTables]:
    """Per-shard tables of one step (gdn_pack_step)."""
    n = len(entries)
    total = sum(e.n_tokens for e in entries)
    ns = np.zeros(n_shards, np.int32)
    nt = np.zeros(n_shards, np.int32)
    slots = np.zeros(max(n, 1), np.int32)
    cu = np.zeros(n + n_shards, np.int32)
    rows = np.zeros(max(total, 1), np.int32)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    abi.call("gdn_pack_step", _entries_c(entries), n, n_shards, slots_per_shard, vp(ns), vp(nt), vp(slots), vp(cu),
             vp(rows))
    out, sb, cb, rb = [], 0, 0, 0
    for s in range(n_shards):
        k, t = int(ns[s]), int(nt[s])
        mine = [e for e in entries if e.slot // slots_per_shard == s]
        reset = np.array([e.slot - s * slots_per_shard for e in mine if e.kind == PREFILL_FIRST], np.int32)
        local = slots[sb:sb + k].copy()
        # gdn_pack_step keeps the step's entry order within a shard, so `mine` lines up with `local`
        if not np.array_equal(local, np.array([e.slot - s * slots_per_shard for e in mine], np.int32)):
            raise RuntimeError("gdn_pack_step reordered a shard's sequences")
        pos = np.array([e.pos for e in mine], np.int32)
        out.append(ShardTables(s, local, cu[cb:cb + k + 1].copy(), rows[rb:rb + t].copy(), reset, pos))
        sb, cb, rb = sb + k, cb + k + 1, rb + t
    return out


class TokenScheduler:
    """Continuous-batching scheduler over sharded pool slots (C++: gdn_sched_*)."""

    def __init__(self, max_batch: int, n_shards: int = 1, slots_per_shard: int = 256, prefill_budget: int = 1,
                 prefill_chunk: int = 0):
        self.n_shards = n_shards
        self.slots_per_shard = slots_per_shard
        cfg = abi.GdnSchedConfigC(n_shards, slots_per_shard, max_batch, prefill_budget, prefill_chunk)
        h = C.c_void_p()
        abi.call("gdn_sched_create", C.byref(cfg), C.byref(h))
        self.h = h
        self._cap = 0
        self._entries = None
        self._n_planned = 0

    def close(self):
        if getattr(self, "h", None):
            abi.lib().gdn_sched_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def enqueue(self, prompt_len: int, max_tokens: int) -> int:
        sid = C.c_uint64()
        abi.call("gdn_sched_enqueue", self.h, prompt_len, max_tokens, C.byref(sid))
        return int(sid.value)

    def plan(self) -> list[StepEntry]:
        st = self.stats
        cap = st["prefilling"] + st["waiting"] + st["active"] + 1
        if cap > self._cap:
            self._cap = 2 * cap
            self._entries = (abi.GdnStepEntryC * self._cap)()
        n = C.c_int32()
        abi.call("gdn_sched_plan", self.h, self._entries, self._cap, C.byref(n))
        self._n_planned = n.value
        return [StepEntry(int(e.seq_id), e.slot, e.n_tokens, e.kind, e.pos) for e in self._entries[:n.value]]

    def complete(self, stop=None):
        """stop[i]: entry i of the last plan produced an end token (default: none did)."""
        flags = np.zeros(max(self._n_planned, 1), np.uint8)
        if stop is not None:
            flags[:self._n_planned] = np.asarray(stop, bool)[:self._n_planned]
        abi.call("gdn_sched_complete", self.h, flags.ctypes.data_as(C.c_void_p))
        self._n_planned = 0

    def drain_finished(self) -> list[tuple[int, int]]:
        out = []
        ids = (C.c_uint64 * 256)()
        rs = (C.c_int32 * 256)()
        n = C.c_int32()
        while True:
            abi.call("gdn_sched_drain_finished", self.h, ids, rs, 256, C.byref(n))
            out += [(int(ids[i]), int(rs[i])) for i in range(n.value)]
            if n.value < 256:
                return out

    @property
    def stats(self) -> dict:
        s = abi.GdnSchedStatsC()
        abi.call("gdn_sched_stats_get", self.h, C.byref(s))
        return {k: int(getattr(s, k)) for k, _ in abi.GdnSchedStatsC._fields_}

    def active_ids(self) -> list[int]:
        n_act = self.stats["active"]
        ids = (C.c_uint64 * max(n_act, 1))()
        n = C.c_int32()
        abi.call("gdn_sched_active_ids", self.h, ids, n_act, C.byref(n))
        return [int(ids[i]) for i in range(n.value)]

    def free_slots(self, shard: int) -> int:
        n = C.c_int32()
        abi.call("gdn_sched_free_slots", self.h, shard, C.byref(n))
        return n.value

    def has_work(self) -> bool:
        s = self.stats
        return s["waiting"] + s["prefilling"] + s["active"] > 0

    def pending_count(self) -> int:
        s = self.stats
        return s["waiting"] + s["prefilling"] + s["active"]


class StackExecutor:
    """Runs planned steps of the residual GDN stack on one GPU's pool (one shard).

    ``weights``: one ``gdn.MixerWeights`` per pool layer.  ``step`` takes the shard's tables
    and its rows ``h`` ([n_tokens, hidden] bf16 on the pool's device, updated in place).
    """

    def __init__(self, pool, weights, max_batch_size: int = 256):
        import torch
        self.pool = pool
        self.weights = weights
        self._max_batch = max_batch_size
        self.device = torch.device(f"cuda:{pool.device}")
        self.stream = torch.cuda.Stream(self.device)
        self._event = None

    def max_batch_size(self) -> int:
        return self._max_batch

    def supports_pipeline(self) -> bool:
        return True

    def submit(self, tables: ShardTables, h):
        """Reset newly admitted slots and launch the stack on the executor's stream (asynchronous)."""
        import torch
        if tables.n_tokens == 0:
            return
        self.pool.reserve_tokens(tables.n_tokens)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            slot_ids = torch.from_numpy(tables.slot_ids).to(self.device, non_blocking=True)
            cu = torch.from_numpy(tables.cu_seqlens).to(self.device, non_blocking=True)
            if tables.reset_slots.size:
                self.pool.reset(tables.reset_slots, stream=self.stream)
            self.pool.stack_step(self.weights, h, slot_ids, cu, tables.n_tokens, stream=self.stream)
            self._event = torch.cuda.Event()
            self._event.record(self.stream)
            h.record_stream(self.stream)

    def collect(self):
        """Wait for the last submitted step (collect_batch)."""
        if self._event is not None:
            self._event.synchronize()
            self._event = None

    def step(self, tables: ShardTables, h):
        self.submit(tables, h)
        self.collect()


def run_sharded_step(entries, shards: list[ShardTables], rows, run_local, dist, rank: int, world: int):
    """One planned step over ``world`` ranks, rank r owning shard r.

    Rank 0 holds the step's packed input ``rows`` ([total, hidden] host tensor) and receives
    every shard's output rows back into it; ``run_local(tables, x) -> y`` runs this rank's
    shard (x, y host tensors [n_tokens, hidden]).  Other ranks pass ``rows=None``.
    Every rank calls this with the same ``entries`` / ``shards``.
    """
    import torch
    mine = shards[rank]
    meta = [rows.shape[1], str(rows.dtype)] if rank == 0 else [None, None]
    dist.broadcast_object_list(meta, src=0)
    hidden = meta[0]
    dtype = getattr(torch, meta[1].split(".")[-1])
    if rank == 0:
        for r in range(1, world):
            if shards[r].n_tokens:
                dist.send(rows[torch.from_numpy(shards[r].row_src).long()].contiguous(), dst=r)
        x = rows[torch.from_numpy(mine.row_src).long()].contiguous() if mine.n_tokens else None
    else:
        x = None
        if mine.n_tokens:
            x = torch.empty((mine.n_tokens, hidden), dtype=dtype)
            dist.recv(x, src=0)
    y = run_local(mine, x) if mine.n_tokens else None
    if rank == 0:
        if mine.n_tokens:
            rows[torch.from_numpy(mine.row_src).long()] = y
        for r in range(1, world):
            if shards[r].n_tokens:
                buf = torch.empty((shards[r].n_tokens, hidden), dtype=dtype)
                dist.recv(buf, src=r)
                rows[torch.from_numpy(shards[r].row_src).long()] = buf
    elif mine.n_tokens:
        dist.send(y.contiguous(), dst=0)
