"""GPU parity in the shape of config 5 (sharded serving): live sequences sit in two slot-range shards of 64
slots each (global slot g belongs to shard g // 64, local slot g % 64).  Every step all of them advance, a
seeded 10% with a prefill chunk of U[64, 320] tokens and the rest one decode token, in a random global order.
The host packer (gdn_pack_step) splits each step into per-shard tables (local slots, cu_seqlens and the rows
each shard takes from the step's packed input); each shard's pool runs its own call (both shards on one GPU
here; in serving, one shard per GPU with no exchange), and the outputs put back by row must match the oracle
run on the whole step.  One full-width GDN layer, three steps, prior state in every slot."""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def sched(pkg):
    return importlib.import_module("qwen_mlx_b200.sched")


def test_config5_shaped_sharded_steps(gdn, synth, oracle, sched):
    cfg = synth.GdnConfig(n_layers=1)
    rng = np.random.default_rng(5)
    per, n_shards, n_live = 64, 2, 40
    gslots = rng.permutation(per * n_shards)[:n_live]
    assert len({int(g) // per for g in gslots}) == n_shards
    conv, rec = synth.random_states(cfg, n_live, seed=55, tag="cfg5")
    conv, rec = conv.copy(), rec.copy()
    w = synth.layer_weights(cfg, 0, with_proj=False)
    f = synth.bf16_to_f32
    pools = [gdn.StatePool(cfg, n_slots=per, device=0) for _ in range(n_shards)]
    try:
        lw = gdn.LayerWeights(w, DEV)
        for i, g in enumerate(gslots):
            pools[int(g) // per].import_(int(g) % per, 0, rec[i], conv[i])
        for step in range(3):
            order = rng.permutation(n_live)          # packing order of the step (sequence indices)
            lens = np.ones(n_live, np.int64)
            n_pref = max(1, int(round(0.1 * n_live)))
            lens[:n_pref] = rng.integers(64, 321, n_pref)
            lens = lens[rng.permutation(n_live)]     # chunks land anywhere in the packing
            entries = [sched.StepEntry(int(i), int(gslots[i]), int(n), sched.DECODE if n == 1 else sched.PREFILL_CONT,
                                       1000) for i, n in zip(order, lens)]
            cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
            N = int(cu[-1])
            inp = synth.step_inputs(cfg, N, seed=500 + step, tag="cfg5")
            out = np.zeros((N, cfg.z_dim), np.uint16)
            tables = sched.pack_step(entries, n_shards, per)
            assert sorted(np.concatenate([t.row_src for t in tables]).tolist()) == list(range(N))
            for t in tables:
                if t.n_seq == 0:
                    continue
                rows = t.row_src
                pool = pools[t.shard]
                o = torch.empty((t.n_tokens, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
                pool.reserve_tokens(t.n_tokens)
                pool.layer_step(0, lw, gdn.bf16_to_device(inp["qkv"][rows], DEV),
                                gdn.bf16_to_device(inp["z"][rows], DEV), gdn.bf16_to_device(inp["ab"][rows], DEV), o,
                                torch.from_numpy(t.slot_ids).to(DEV), torch.from_numpy(t.cu_seqlens).to(DEV),
                                t.n_tokens)
                torch.cuda.synchronize()
                out[rows] = gdn.bf16_to_host(o)
            ref_out, c2, r2, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv[order], rec[order], cu)
            conv[order], rec[order] = c2, r2
            assert rel_l2(f(out), f(ref_out)) < TOL, f"step {step}"
        for p in pools:
            assert p.check() == 0
        got = [pools[int(g) // per].export(int(g) % per, 0) for g in gslots]
    finally:
        for p in pools:
            p.close()
    assert rel_l2(np.stack([g[0] for g in got]), rec) < TOL
    assert np.array_equal(np.stack([g[1] for g in got]), conv)
