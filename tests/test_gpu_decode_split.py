"""GPU parity of the split decode kernel (gdn_split.cu: each (sequence, v-head) state tile split by
dv rows over 4 CTAs of a cluster), the default for decode-only calls of fewer than 64 sequences.

Covers batched decode at several batch sizes against the oracle, the three decode kernels against
each other, multi-step chains, decode-only calls that carry a 2-token and an empty segment, the
early routing of GDN_STEP_TABLES_STABLE across layers, and the failure detection of its bounded
wait: a test-only control makes one CTA's state wait run out (a copy that is never issued), the
kernel records 1 << 7 and returns, and the next normal call is correct.  Tolerance: rel-L2 1e-3 on
outputs and states; conv states exact.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")
SPLIT, FUSED, TWO_KERNEL = 1, 2, 3


@pytest.fixture
def modes(abi):
    """Restores the default kernel selection and the normal wait bound after each test."""
    lib = abi.lib()

    def set_mode(m):
        assert lib.gdn_set_decode_kernel(m) == abi.GDN_OK
    yield set_mode
    assert lib.gdn_set_decode_kernel(0) == abi.GDN_OK
    assert lib.gdn_test_set_wait_fault(-1, 2_000_000_000) == abi.GDN_OK


def _cu(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


class Layer:
    def __init__(self, gdn, synth, n_slots, n_layers=1):
        self.gdn, self.synth = gdn, synth
        self.cfg = synth.GdnConfig(n_layers=n_layers)
        self.pool = gdn.StatePool(self.cfg, n_slots=n_slots, device=0)
        self.ws = [synth.layer_weights(self.cfg, l, with_proj=False) for l in range(n_layers)]
        self.lws = [gdn.LayerWeights(w, DEV) for w in self.ws]

    def step(self, layer, inp, slots, cu, flags=0):
        g = self.gdn
        N = int(cu[-1])
        out = torch.full((max(N, 1), self.cfg.z_dim), float("nan"), dtype=torch.bfloat16, device=DEV)
        self.pool.layer_step(layer, self.lws[layer], g.bf16_to_device(inp["qkv"], DEV),
                             g.bf16_to_device(inp["z"], DEV), g.bf16_to_device(inp["ab"], DEV), out,
                             torch.from_numpy(np.asarray(slots, np.int32)).to(DEV),
                             torch.from_numpy(np.asarray(cu, np.int32)).to(DEV), N, flags=flags)
        torch.cuda.synchronize()
        return g.bf16_to_host(out[:N])

    def load(self, layer, slots, conv, rec):
        for i, s in enumerate(slots):
            self.pool.import_(int(s), layer, rec[i], conv[i])

    def states(self, layer, slots):
        got = [self.pool.export(int(s), layer) for s in slots]
        return np.stack([g[1] for g in got]), np.stack([g[0] for g in got])

    def close(self):
        self.pool.close()


@pytest.mark.parametrize("B", [1, 2, 8, 33, 63])
def test_split_decode_matches_oracle_over_steps(gdn, synth, oracle, modes, B):
    modes(SPLIT)
    n_slots = B + 5
    L = Layer(gdn, synth, n_slots)
    try:
        cfg = L.cfg
        slots = np.random.default_rng(B).permutation(n_slots)[:B].astype(np.int32)
        cu = _cu([1] * B)
        conv, rec = synth.random_states(cfg, B, seed=3, tag=f"split{B}")
        L.load(0, slots, conv, rec)
        f = synth.bf16_to_f32
        for it in range(3):
            inp = synth.step_inputs(cfg, B, seed=10 + it, tag=f"split{B}")
            out = L.step(0, inp, slots, cu)
            ref_out, conv, rec, _ = oracle.layer_step(cfg, L.ws[0], inp["qkv"], inp["z"], inp["ab"], conv, rec, cu)
            assert rel_l2(f(out), f(ref_out)) < TOL, f"step {it}: output"
            gc, gr = L.states(0, slots)
            assert rel_l2(gr, rec) < TOL, f"step {it}: states"
            assert np.array_equal(gc, conv), f"step {it}: conv states"
        assert L.pool.check() == 0
    finally:
        L.close()


@pytest.mark.parametrize("B", [8, 80])
def test_decode_kernels_agree(gdn, synth, oracle, modes, B):
    """Split, fused and two-kernel decode steps on the same inputs: each within tolerance of the oracle,
    conv states identical."""
    cfg = synth.GdnConfig(n_layers=1)
    slots = (np.arange(B, dtype=np.int32) * 5 + 1) % (B + 3)
    cu = _cu([1] * B)
    conv0, rec0 = synth.random_states(cfg, B, seed=4, tag=f"agree{B}")
    inp = synth.step_inputs(cfg, B, seed=4, tag=f"agree{B}")
    w = synth.layer_weights(cfg, 0, with_proj=False)
    ref_out, ref_conv, ref_rec, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
    f = synth.bf16_to_f32
    for m in (SPLIT, FUSED, TWO_KERNEL):
        modes(m)
        L = Layer(gdn, synth, B + 3)
        try:
            L.load(0, slots, conv0, rec0)
            out = L.step(0, inp, slots, cu)
            gc, gr = L.states(0, slots)
            assert rel_l2(f(out), f(ref_out)) < TOL, f"mode {m}: output"
            assert rel_l2(gr, ref_rec) < TOL, f"mode {m}: states"
            assert np.array_equal(gc, ref_conv), f"mode {m}: conv states"
        finally:
            L.close()


def test_split_decode_only_call_with_two_token_and_empty_segments(gdn, synth, oracle, modes):
    """n_tokens == n_seq does not mean every segment has one token: [2, 0, 1, 1] runs the split kernel's
    per-token loop (f32 conv1d rounding for the 2-token segment) and skips the empty one."""
    modes(SPLIT)
    lens = [2, 0, 1, 1]
    cu = _cu(lens)
    slots = np.array([3, 0, 6, 1], np.int32)
    L = Layer(gdn, synth, 8)
    try:
        cfg = L.cfg
        conv, rec = synth.random_states(cfg, len(lens), seed=6, tag="split_ragged")
        L.load(0, slots, conv, rec)
        inp = synth.step_inputs(cfg, int(cu[-1]), seed=6, tag="split_ragged")
        out = L.step(0, inp, slots, cu)
        ref_out, ref_conv, ref_rec, _ = oracle.layer_step(cfg, L.ws[0], inp["qkv"], inp["z"], inp["ab"], conv, rec, cu)
        f = synth.bf16_to_f32
        assert rel_l2(f(out), f(ref_out)) < TOL
        gc, gr = L.states(0, slots)
        for i in range(len(lens)):
            assert rel_l2(gr[i], ref_rec[i]) < TOL, f"state {i}"
        assert np.array_equal(gc, ref_conv)
        assert L.pool.check() == 0
    finally:
        L.close()


def test_split_stable_tables_across_layers_identical(gdn, synth, abi, modes):
    """Layers 2..L of a step with GDN_STEP_TABLES_STABLE (routing, state slice and windows read before the
    kernel's dependency wait) give the same bytes as plain calls."""
    modes(SPLIT)
    B, n_layers = 8, 4
    slots = np.arange(B, dtype=np.int32)[::-1].copy()
    cu = _cu([1] * B)
    results = []
    for flags in (0, abi.GDN_STEP_TABLES_STABLE):
        L = Layer(gdn, synth, B, n_layers=n_layers)
        try:
            cfg = L.cfg
            for l in range(n_layers):
                conv, rec = synth.random_states(cfg, B, seed=20 + l, tag="stable")
                L.load(l, slots, conv, rec)
            outs = []
            for it in range(2):
                for l in range(n_layers):
                    inp = synth.step_inputs(cfg, B, seed=100 * it + l, tag="stable")
                    outs.append(L.step(l, inp, slots, cu, flags=flags if l else 0))
            states = [L.states(l, slots) for l in range(n_layers)]
            results.append((outs, states))
        finally:
            L.close()
    (o0, s0), (o1, s1) = results
    for a, b in zip(o0, o1):
        assert np.array_equal(a, b)
    for (c0, r0), (c1, r1) in zip(s0, s1):
        assert np.array_equal(c0, c1) and np.array_equal(r0, r1)


def test_split_bounded_wait_reports_timeout_and_next_call_is_correct(gdn, synth, oracle, abi, modes):
    """Failure detection without a GPU fault: CTA 0's state copy is never issued (test-only control), its
    wait runs out after 1 ms, the kernel records 1 << 7 in the pool's error word and returns; the other
    CTAs finish normally.  The next call, with the normal bound, matches the oracle run from the states
    the pool holds after the failed call."""
    modes(SPLIT)
    B = 8
    slots = np.arange(B, dtype=np.int32)
    cu = _cu([1] * B)
    L = Layer(gdn, synth, B)
    try:
        cfg = L.cfg
        conv, rec = synth.random_states(cfg, B, seed=7, tag="timeout")
        L.load(0, slots, conv, rec)
        lib = abi.lib()
        assert lib.gdn_test_set_wait_fault(0, 1_000_000) == abi.GDN_OK
        inp = synth.step_inputs(cfg, B, seed=7, tag="timeout")
        L.step(0, inp, slots, cu)
        assert lib.gdn_test_set_wait_fault(-1, 2_000_000_000) == abi.GDN_OK
        flags = L.pool.check()
        assert flags & (1 << 7), f"error word {flags:#x}: the timeout was not reported"
        # CTA 0 serves sequence 0, v-head 0, rows 0..31: those rows kept their old values
        _, rec_after = L.states(0, slots)
        assert np.array_equal(rec_after[0, 0, :32], rec[0, 0, :32])
        # the next call is normal
        conv_now, rec_now = L.states(0, slots)
        inp2 = synth.step_inputs(cfg, B, seed=8, tag="timeout")
        out = L.step(0, inp2, slots, cu)
        assert L.pool.check() == 0
        ref_out, ref_conv, ref_rec, _ = oracle.layer_step(cfg, L.ws[0], inp2["qkv"], inp2["z"], inp2["ab"],
                                                          conv_now, rec_now, cu)
        f = synth.bf16_to_f32
        assert rel_l2(f(out), f(ref_out)) < TOL
        gc, gr = L.states(0, slots)
        assert rel_l2(gr, ref_rec) < TOL
        assert np.array_equal(gc, ref_conv)
    finally:
        L.close()


def test_decode_kernel_mode_is_validated(abi):
    lib = abi.lib()
    assert lib.gdn_set_decode_kernel(4) == abi.GDN_E_INVALID
    assert lib.gdn_test_set_wait_fault(-1, 0) == abi.GDN_E_INVALID


@pytest.mark.parametrize("mode,lens", [(SPLIT, [1] * 8), (FUSED, [1] * 70), (TWO_KERNEL, [1] * 8),
                                       (0, [1, 5, 40, 1, 130])])
def test_bf16_dt_bias_gates_in_every_kernel(gdn, synth, oracle, modes, mode, lens):
    """A layer whose dt_bias is stored in bf16 (dt_bias_bf16): every decode kernel and the prefill path
    (prep + chunked kernel for segments of >= 32 tokens) round a + dt_bias and its exp to bf16 as the
    reference does (compiled_ops.rs:36-37); outputs and states match the oracle's bf16 mode."""
    modes(mode)
    cfg = synth.GdnConfig(n_layers=1)
    n = len(lens)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    w["dt_bias"] = synth.bf16_to_f32(synth.f32_to_bf16(w["dt_bias"]))
    w["dt_bias_bf16"] = True
    cu = _cu(lens)
    slots = np.arange(n, dtype=np.int32)[::-1].copy()
    conv0, rec0 = synth.random_states(cfg, n, seed=9, tag="dt16")
    inp = synth.step_inputs(cfg, int(cu[-1]), seed=9, tag="dt16")
    L = Layer(gdn, synth, n + 2)
    try:
        L.ws[0] = w
        L.lws[0] = gdn.LayerWeights(w, DEV)
        L.load(0, slots, conv0, rec0)
        out = L.step(0, inp, slots, cu)
        ref_out, ref_conv, ref_rec, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
        w32 = dict(w, dt_bias_bf16=False)
        f32_out = oracle.layer_step(cfg, w32, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)[0]
        f = synth.bf16_to_f32
        r = rel_l2(f(out), f(ref_out))
        assert r < TOL
        assert r < 0.5 * rel_l2(f(f32_out), f(ref_out)), "the bf16 gate rounding is not what the kernels did"
        gc, gr = L.states(0, slots)
        assert rel_l2(gr, ref_rec) < TOL
        assert np.array_equal(gc, ref_conv)
        assert L.pool.check() == 0
    finally:
        L.close()
