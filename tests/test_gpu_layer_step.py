"""GPU parity of the fused layer step (gdn_layer_step) against the oracle.

Covers batched decode, ragged packed prefill + decode with scrambled slot ids,
empty sequences, the committed golden layer cases, multi-step chains, bit-exact
routing (results independent of which slot holds a sequence), and the kernel's
own bounds checks.  Tolerance: rel-L2 1e-3 on outputs and states; conv states
(copies of bf16 inputs) must match exactly.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")


class Harness:
    """A pool + one layer's weights + device copies of a packed batch."""

    def __init__(self, gdn, synth, cfg, n_slots, layer_seed=0):
        self.gdn, self.synth, self.cfg = gdn, synth, cfg
        self.pool = gdn.StatePool(cfg, n_slots=n_slots, device=0)
        self.w = synth.layer_weights(cfg, layer_seed, with_proj=False)
        self.lw = gdn.LayerWeights(self.w, DEV)

    def load_states(self, layer, slots, conv, rec):
        for i, s in enumerate(slots):
            self.pool.import_(int(s), layer, rec[i], conv[i])

    def step(self, layer, inp, slots, cu):
        g = self.gdn
        N = int(cu[-1])
        out = torch.full((max(N, 1), self.cfg.z_dim), float("nan"), dtype=torch.bfloat16, device=DEV)
        self.pool.layer_step(layer, self.lw, g.bf16_to_device(inp["qkv"], DEV), g.bf16_to_device(inp["z"], DEV),
                             g.bf16_to_device(inp["ab"], DEV), out, torch.from_numpy(np.asarray(slots, np.int32)).to(DEV),
                             torch.from_numpy(np.asarray(cu, np.int32)).to(DEV), N)
        torch.cuda.synchronize()
        return g.bf16_to_host(out[:N])

    def states(self, layer, slots):
        conv, rec = [], []
        for s in slots:
            r, c = self.pool.export(int(s), layer)
            rec.append(r)
            conv.append(c)
        return np.stack(conv), np.stack(rec)

    def close(self):
        self.pool.close()


@pytest.fixture
def H(gdn, synth):
    hs = []

    def make(cfg=None, n_slots=16):
        h = Harness(gdn, synth, cfg or synth.GdnConfig(n_layers=2), n_slots)
        hs.append(h)
        return h
    yield make
    for h in hs:
        h.close()


def _cu(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def _compare(synth, got_out, ref_out, got_states, ref_states, lens=None):
    f = synth.bf16_to_f32
    if got_out.size:
        assert rel_l2(f(got_out), f(ref_out)) < TOL
    gc, gr = got_states
    rc, rr = ref_states
    for i in range(len(gr)):
        if lens is not None and lens[i] == 0:
            continue
        assert rel_l2(gr[i], rr[i]) < TOL, f"state {i}"
    assert np.array_equal(gc, rc), "conv state"


@pytest.mark.parametrize("B", [1, 8, 33, 64, 129])
def test_decode_batch(H, synth, oracle, B):
    """B < 64: prep kernel + recurrence kernel; B >= 64: the fused one-kernel decode step."""
    h = H(n_slots=max(B, 16) + 3)
    cfg = h.cfg
    lens = [1] * B
    cu = _cu(lens)
    slots = (np.arange(B, dtype=np.int32) * 7 + 2) % (max(B, 16) + 3)
    assert len(set(slots.tolist())) == B
    inp = synth.step_inputs(cfg, B, seed=1, tag=f"dec{B}")
    conv0, rec0 = synth.random_states(cfg, B, seed=1, tag=f"dec{B}")
    h.load_states(1, slots, conv0, rec0)
    out = h.step(1, inp, slots, cu)
    assert h.pool.check() == 0
    ref = oracle.layer_step(cfg, h.w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
    _compare(synth, out, ref[0], h.states(1, slots), (ref[1], ref[2]))


@pytest.mark.parametrize("lens", [[0, 2, 1, 1], [6, 0, 0, 0, 0, 0], [1, 0, 9, 0, 1, 0, 0, 0, 0, 1, 0, 0],
                                  [1] * 60 + [0, 2, 0, 6, 0, 0, 0, 0], [0] * 40 + [1] * 23 + [41]])
def test_decode_call_with_uneven_segments(H, synth, oracle, lens):
    """Calls with n_tokens == n_seq take a decode path (the fused kernel from 64 sequences on); it must
    also handle empty segments and multi-token segments (past the 4th token their records go through
    the scratch)."""
    n_slots = max(16, len(lens) + 3)
    h = H(n_slots=n_slots)
    cfg = h.cfg
    assert sum(lens) == len(lens)
    cu = _cu(lens)
    slots = np.array([(5 * i + 3) % n_slots for i in range(len(lens))], np.int32)
    assert len(set(slots.tolist())) == len(lens)
    inp = synth.step_inputs(cfg, int(cu[-1]), seed=4, tag=f"uneven{len(lens)}")
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=4, tag=f"uneven{len(lens)}")
    h.load_states(1, slots, conv0, rec0)
    out = h.step(1, inp, slots, cu)
    assert h.pool.check() == 0
    ref = oracle.layer_step(cfg, h.w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
    _compare(synth, out, ref[0], h.states(1, slots), (ref[1], ref[2]), lens)
    for i, n in enumerate(lens):
        if n == 0:
            r, c = h.pool.export(int(slots[i]), 1)
            assert np.array_equal(r, rec0[i]) and np.array_equal(c, conv0[i])


def test_ragged_prefill_and_decode_scrambled(H, synth, oracle):
    h = H(n_slots=24)
    cfg = h.cfg
    lens = [1, 3, 1, 5, 0, 2, 17, 1, 64]
    cu = _cu(lens)
    slots = np.array([20, 3, 7, 0, 9, 14, 6, 23, 1], np.int32)
    inp = synth.step_inputs(cfg, int(cu[-1]), seed=2, tag="rag")
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=2, tag="rag")
    h.load_states(0, slots, conv0, rec0)
    out = h.step(0, inp, slots, cu)
    assert h.pool.check() == 0
    ref = oracle.layer_step(cfg, h.w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
    _compare(synth, out, ref[0], h.states(0, slots), (ref[1], ref[2]), lens)
    # the empty sequence's state is untouched, bit for bit
    r, c = h.pool.export(9, 0)
    assert np.array_equal(r, rec0[4]) and np.array_equal(c, conv0[4])


def test_golden_layer_cases(H, synth, gdn):
    gdir = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(gdir))
    import make_golden as mg
    manifest = json.loads((gdir / "manifest.json").read_text())
    samples = np.load(gdir / "golden.npz")
    stride = manifest["sample_stride"]
    f = synth.bf16_to_f32
    for case in mg.LAYER_CASES:
        cfg, w, inp, conv, rec, cu = mg.layer_case_inputs(case)
        h = H(cfg=synth.GdnConfig(n_layers=1), n_slots=len(case["lens"]))
        slots = np.arange(len(case["lens"]), dtype=np.int32)[::-1].copy()
        h.load_states(0, slots, conv, rec)
        out = h.step(0, inp, slots, cu)
        gc, gr = h.states(0, slots)
        name = case["name"]
        assert rel_l2(f(out.reshape(-1)[::stride]), f(samples[name + "/out"])) < TOL, name
        assert rel_l2(gr.reshape(-1)[::stride], samples[name + "/rec"]) < TOL, name
        assert np.array_equal(gc.reshape(-1)[::stride], samples[name + "/conv"]), name


def test_multi_step_chain_two_layers(H, synth, oracle):
    """Prefill (zero state) then decode steps, on two layers with distinct weights."""
    cfg = synth.GdnConfig(n_layers=2)
    h = H(cfg=cfg, n_slots=8)
    h1 = Harness(h.gdn, synth, cfg, 1, layer_seed=1)   # second layer's weights
    try:
        slots = np.array([5, 2, 7], np.int32)
        n = len(slots)
        conv = [np.zeros((n, 3, cfg.conv_dim), np.uint16) for _ in range(2)]
        rec = [np.zeros((n, cfg.hv, 128, 128), np.float32) for _ in range(2)]
        schedule = [[7, 1, 12], [1, 1, 1], [1, 4, 1], [1, 1, 1]]
        for it, lens in enumerate(schedule):
            cu = _cu(lens)
            for layer, hw in ((0, h), (1, h1)):
                inp = synth.step_inputs(cfg, int(cu[-1]), seed=100 + it, tag=f"chain{layer}")
                hw_pool = h.pool
                N = int(cu[-1])
                out_t = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
                g = h.gdn
                hw_pool.layer_step(layer, hw.lw, g.bf16_to_device(inp["qkv"], DEV), g.bf16_to_device(inp["z"], DEV),
                                   g.bf16_to_device(inp["ab"], DEV), out_t, torch.from_numpy(slots).to(DEV),
                                   torch.from_numpy(cu).to(DEV), N)
                torch.cuda.synchronize()
                ref_out, conv[layer], rec[layer], _ = oracle.layer_step(cfg, hw.w, inp["qkv"], inp["z"], inp["ab"],
                                                                        conv[layer], rec[layer], cu)
                assert rel_l2(synth.bf16_to_f32(g.bf16_to_host(out_t)), synth.bf16_to_f32(ref_out)) < TOL
        for layer in range(2):
            gc, gr = h.states(layer, slots)
            assert np.array_equal(gc, conv[layer])
            assert rel_l2(gr, rec[layer]) < TOL
    finally:
        h1.close()


def test_routing_is_bit_exact_across_slot_assignments(H, synth):
    """The same sequences in different slots give byte-identical outputs and states."""
    h = H(n_slots=32)
    cfg = h.cfg
    lens = [1, 4, 1, 2, 1]
    cu = _cu(lens)
    inp = synth.step_inputs(cfg, int(cu[-1]), seed=3, tag="route")
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=3, tag="route")
    sa = np.array([0, 1, 2, 3, 4], np.int32)
    sb = np.array([31, 17, 8, 22, 5], np.int32)
    h.load_states(0, sa, conv0, rec0)
    h.load_states(0, sb, conv0, rec0)
    out_a = h.step(0, inp, sa, cu)
    out_b = h.step(0, inp, sb, cu)
    assert np.array_equal(out_a, out_b)
    ca, ra = h.states(0, sa)
    cb, rb = h.states(0, sb)
    assert np.array_equal(ra.view(np.uint32), rb.view(np.uint32))
    assert np.array_equal(ca, cb)


def test_export_import_round_trip_and_reset(H, synth):
    h = H(n_slots=4)
    cfg = h.cfg
    conv0, rec0 = synth.random_states(cfg, 1, seed=4, tag="rt")
    h.pool.import_(2, 1, rec0[0], conv0[0])
    r, c = h.pool.export(2, 1)
    assert np.array_equal(r.view(np.uint32), rec0[0].view(np.uint32)) and np.array_equal(c, conv0[0])
    h.pool.reset([2])
    torch.cuda.synchronize()
    r, c = h.pool.export(2, 1)
    assert not r.any() and not c.any()


def test_device_bounds_check_skips_bad_slot(H, synth, oracle):
    """An out-of-range slot id in a device table is skipped and reported; other sequences still run."""
    h = H(n_slots=8)
    cfg = h.cfg
    lens = [1, 1]
    cu = _cu(lens)
    slots = np.array([3, 99], np.int32)   # 99 is outside [0, 8): the kernel's own check rejects it
    inp = synth.step_inputs(cfg, 2, seed=5, tag="bad")
    conv0, rec0 = synth.random_states(cfg, 2, seed=5, tag="bad")
    h.load_states(0, [3], conv0[:1], rec0[:1])
    out = h.step(0, inp, slots, cu)
    flags = h.pool.check()
    assert flags & (1 << 3)
    assert h.pool.check() == 0          # cleared by the previous read
    ref = oracle.layer_step(cfg, h.w, inp["qkv"][:1], inp["z"][:1], inp["ab"][:1], conv0[:1], rec0[:1], cu[:2])
    assert rel_l2(synth.bf16_to_f32(out[:1]), synth.bf16_to_f32(ref[0])) < TOL


@pytest.mark.parametrize("B", [8, 33, 80])
def test_stable_tables_flag_gives_identical_results(gdn, synth, B):
    """gdn_layer_step_ex with GDN_STEP_TABLES_STABLE (layers 2..L of a step read routing and windows early)
    computes exactly what gdn_layer_step computes: outputs and states byte-identical over a 4-layer,
    3-step decode chain with scrambled slots."""
    import importlib
    abi = importlib.import_module("qwen_mlx_b200.abi")
    cfg = synth.GdnConfig(n_layers=4)
    rng = np.random.default_rng(11)
    slots = rng.permutation(128)[:B].astype(np.int32)
    cu = np.arange(B + 1, dtype=np.int32)
    ws = [gdn.LayerWeights(synth.layer_weights(cfg, l, with_proj=False), DEV) for l in range(cfg.n_layers)]
    conv0, rec0 = synth.random_states(cfg, B, seed=21, tag="stable")
    results = []
    for use_flag in (False, True):
        outs = []
        with gdn.StatePool(cfg, n_slots=128, device=0) as pool:
            for l in range(cfg.n_layers):
                for i in range(B):
                    pool.import_(int(slots[i]), l, rec0[i], conv0[i])
            sd, cd = torch.from_numpy(slots).to(DEV), torch.from_numpy(cu).to(DEV)
            for step in range(3):
                for l in range(cfg.n_layers):
                    inp = synth.step_inputs(cfg, B, seed=70 + 10 * step + l, tag="stable")
                    out = torch.empty((B, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
                    pool.layer_step(l, ws[l], gdn.bf16_to_device(inp["qkv"], DEV), gdn.bf16_to_device(inp["z"], DEV),
                                    gdn.bf16_to_device(inp["ab"], DEV), out, sd, cd, B,
                                    flags=abi.GDN_STEP_TABLES_STABLE if (use_flag and l > 0) else 0)
                    outs.append(out)
            torch.cuda.synchronize()
            assert pool.check() == 0
            st = [pool.export(int(s), l) for l in range(cfg.n_layers) for s in slots]
        results.append(([gdn.bf16_to_host(o) for o in outs], st))
    (o0, s0), (o1, s1) = results
    assert all(np.array_equal(a, b) for a, b in zip(o0, o1))
    assert all(np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) for a, b in zip(s0, s1))


def test_layer_step_ex_rejects_unknown_flags(gdn, synth):
    import importlib
    abi = importlib.import_module("qwen_mlx_b200.abi")
    cfg = synth.GdnConfig(n_layers=1)
    w = gdn.LayerWeights(synth.layer_weights(cfg, 0, with_proj=False), DEV)
    with gdn.StatePool(cfg, n_slots=4, device=0) as pool:
        z = torch.zeros((1, 16384), dtype=torch.bfloat16, device=DEV)
        t = torch.zeros(2, dtype=torch.int32, device=DEV)
        with pytest.raises(abi.GdnError) as e:
            pool.layer_step(0, w, z, z, z, z, t[:1], t, 1, flags=0x10)
        assert e.value.code == abi.GDN_E_INVALID
