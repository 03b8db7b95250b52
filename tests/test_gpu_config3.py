"""GPU parity in the shape of config 3 (ragged continuous batching on one GPU): a 256-slot pool
holds 64 live sequences with prior state; every step a seeded 50-100% subset is active, about 10%
of the active ones carry a prefill chunk of U[1, 512] tokens and the rest decode one token, all
packed in one call with scrambled slots.  One full-width GDN layer (Hk 16, Hv 32), five steps; the
oracle runs the same steps on densely gathered states.  Chunks of >= 32 tokens take the chunked
tensor-core path, shorter ones the token-sequential kernel, decode tokens either the two-kernel or
the fused decode step, so every path meets inside one call and carries its state to the next."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")


def test_config3_shaped_continuous_batching(gdn, synth, oracle):
    cfg = synth.GdnConfig(n_layers=1)
    rng = np.random.default_rng(3)
    n_live, n_slots = 64, 256
    slots = rng.permutation(n_slots)[:n_live].astype(np.int32)
    conv, rec = synth.random_states(cfg, n_live, seed=33, tag="cfg3")
    conv, rec = conv.copy(), rec.copy()
    w = synth.layer_weights(cfg, 0, with_proj=False)
    f = synth.bf16_to_f32
    paths = set()
    with gdn.StatePool(cfg, n_slots=n_slots, device=0) as pool:
        lw = gdn.LayerWeights(w, DEV)
        for i in range(n_live):
            pool.import_(int(slots[i]), 0, rec[i], conv[i])
        for step in range(5):
            n_act = int(rng.integers(n_live // 2, n_live + 1))
            act = rng.permutation(n_live)[:n_act]
            n_pref = max(1, int(round(0.1 * n_act)))
            lens = np.ones(n_act, np.int64)
            lens[:n_pref] = rng.integers(1, 513, n_pref)
            order = rng.permutation(n_act)          # prefill chunks land anywhere in the packing
            act, lens = act[order], lens[order]
            paths |= {"wy" if n >= 32 else ("seq" if n > 1 else "decode") for n in lens}
            cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
            N = int(cu[-1])
            inp = synth.step_inputs(cfg, N, seed=300 + step, tag="cfg3")
            out = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
            pool.reserve_tokens(N)
            pool.layer_step(0, lw, gdn.bf16_to_device(inp["qkv"], DEV), gdn.bf16_to_device(inp["z"], DEV),
                            gdn.bf16_to_device(inp["ab"], DEV), out, torch.from_numpy(slots[act]).to(DEV),
                            torch.from_numpy(cu).to(DEV), N)
            torch.cuda.synchronize()
            ref_out, c2, r2, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv[act], rec[act], cu)
            conv[act], rec[act] = c2, r2
            assert rel_l2(f(gdn.bf16_to_host(out)), f(ref_out)) < TOL, f"step {step}"
        assert pool.check() == 0
        got = [pool.export(int(s), 0) for s in slots]
    assert paths >= {"wy", "decode"}
    assert rel_l2(np.stack([g[0] for g in got]), rec) < TOL
    assert np.array_equal(np.stack([g[1] for g in got]), conv)
