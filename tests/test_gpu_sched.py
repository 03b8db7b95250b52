"""GPU parity of scheduled serving: the token scheduler drives StackExecutor (slot resets plus
one gdn_stack_step per step over a mixed batch of prompt chunks and decode tokens), and the
oracle runs the same plan with dense per-sequence states.  Two residual layers of a
reduced-width model; tolerance calibrated by the oracle's GEMM-order spread (conftest)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ALT_ORDERS, order_noise, rel_l2, with_order

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")


def test_scheduled_stack_matches_oracle(gdn, synth, oracle, pkg):
    import importlib
    sched = importlib.import_module("qwen_mlx_b200.sched")
    cfg = synth.GdnConfig(hidden=256, n_k_heads=2, n_v_heads=4, n_layers=2)
    L = cfg.n_layers
    ws = [synth.layer_weights(cfg, l, with_proj=True) for l in range(L)]
    rng = np.random.default_rng(5)
    reqs = [(int(rng.integers(1, 100)), int(rng.integers(1, 6))) for _ in range(10)]
    s = sched.TokenScheduler(max_batch=4, n_shards=1, slots_per_shard=6, prefill_budget=2, prefill_chunk=48)
    for p, m in reqs:
        s.enqueue(p, m)

    def zero_state():
        return (np.zeros((L, 3, cfg.conv_dim), np.uint16), np.zeros((L, cfg.hv, 128, 128), np.float32))

    states = {o: {} for o in (0, *ALT_ORDERS)}   # oracle state per sequence, per GEMM order
    got_all, ref_all = [], {o: [] for o in ALT_ORDERS}
    ref0 = []
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=6, device=0) as pool:
        ex = sched.StackExecutor(pool, [gdn.MixerWeights(w, DEV) for w in ws])
        n_steps = 0
        kinds = set()
        while s.has_work():
            entries = s.plan()
            kinds |= {e.kind for e in entries}
            (tables,) = sched.pack_step(entries, 1, 6)
            h0 = np.concatenate([np.stack([synth.normal_bf16(1000 * e.seq_id + e.pos + t, "sched_h", (cfg.hidden,))
                                           for t in range(e.n_tokens)]) for e in entries])
            hd = gdn.bf16_to_device(h0, DEV)
            ex.step(tables, hd)
            got_all.append(f(gdn.bf16_to_host(hd)))
            cu = np.concatenate([[0], np.cumsum([e.n_tokens for e in entries])]).astype(np.int32)
            for o in (0, *ALT_ORDERS):
                st = states[o]
                for e in entries:
                    if e.kind == sched.PREFILL_FIRST:
                        st[e.seq_id] = zero_state()
                cs = np.stack([st[e.seq_id][0] for e in entries], axis=1)
                rs = np.stack([st[e.seq_id][1] for e in entries], axis=1)
                h, cs, rs = with_order(oracle, o, lambda: oracle.stack_step(cfg, ws, h0, cs, rs, cu))
                for i, e in enumerate(entries):
                    st[e.seq_id] = (cs[:, i].copy(), rs[:, i].copy())
                (ref0 if o == 0 else ref_all[o]).append(f(h))
            s.complete([e.seq_id == 3 and e.kind == sched.DECODE for e in entries])
            n_steps += 1
        assert pool.check() == 0
    assert kinds == {sched.DECODE, sched.PREFILL_FIRST, sched.PREFILL_CONT}
    assert n_steps > 5
    got = np.concatenate(got_all)
    ref = np.concatenate(ref0)
    tol = max(TOL, 2 * order_noise(ref, [np.concatenate(ref_all[o]) for o in ALT_ORDERS]))
    assert rel_l2(got, ref) < tol
