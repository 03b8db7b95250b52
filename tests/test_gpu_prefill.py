"""GPU parity of the chunked (WY) prefill path on tcgen05 tensor cores.

Segments of at least 32 tokens in one gdn_layer_step call run the chunked kernel
(64-token chunks, hi/lo bf16 splits of the f32 operands); shorter segments and decode
tokens run the token-sequential kernel in the same call.  Compared with the oracle's
token-sequential recurrence at rel-L2 1e-3 (outputs and states); conv states exactly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
DEV = torch.device("cuda:0")


def _cu(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def _run(gdn, synth, oracle, cfg, w, lens, slots, conv0, rec0, seed, tag, pool=None):
    cu = _cu(lens)
    N = int(cu[-1])
    inp = synth.step_inputs(cfg, N, seed=seed, tag=tag)
    lw = gdn.LayerWeights(w, DEV)
    out = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
    pool.layer_step(0, lw, gdn.bf16_to_device(inp["qkv"], DEV), gdn.bf16_to_device(inp["z"], DEV),
                    gdn.bf16_to_device(inp["ab"], DEV), out, torch.from_numpy(slots).to(DEV),
                    torch.from_numpy(cu).to(DEV), N)
    torch.cuda.synchronize()
    assert pool.check() == 0
    ref = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
    return gdn.bf16_to_host(out), ref


@pytest.mark.parametrize("zero_state", [True, False])
def test_chunked_prefill_ragged(gdn, synth, oracle, zero_state):
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    lens = [32, 1, 64, 65, 3, 127, 200, 333]
    slots = np.array([9, 2, 14, 0, 5, 11, 3, 7], np.int32)
    if zero_state:
        conv0 = np.zeros((len(lens), 3, cfg.conv_dim), np.uint16)
        rec0 = np.zeros((len(lens), cfg.hv, 128, 128), np.float32)
    else:
        conv0, rec0 = synth.random_states(cfg, len(lens), seed=6, tag="wy")
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=16, device=0) as pool:
        pool.reserve_tokens(int(sum(lens)))
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        out, (ref_out, ref_cs, ref_rs, _) = _run(gdn, synth, oracle, cfg, w, lens, slots, conv0, rec0, 6, "wy",
                                                 pool=pool)
        cu = _cu(lens)
        for i, s in enumerate(slots):
            a, b = cu[i], cu[i + 1]
            assert rel_l2(f(out[a:b]), f(ref_out[a:b])) < TOL, f"output of segment {i} (T={lens[i]})"
            r, c = pool.export(int(s), 0)
            assert rel_l2(r, ref_rs[i]) < TOL, f"state of segment {i} (T={lens[i]})"
            assert np.array_equal(c, ref_cs[i]), f"conv state of segment {i}"


def test_chunked_prefill_continuation_then_decode(gdn, synth, oracle):
    """Prompt split over two calls (150 + 90 tokens), then decode steps, on one slot."""
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    slots = np.array([4, 1], np.int32)
    conv = np.zeros((2, 3, cfg.conv_dim), np.uint16)
    rec = np.zeros((2, cfg.hv, 128, 128), np.float32)
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=8, device=0) as pool:
        for it, lens in enumerate([[150, 40], [90, 1], [1, 1], [1, 70]]):
            out, (ref_out, conv, rec, _) = _run(gdn, synth, oracle, cfg, w, lens, slots, conv, rec, 20 + it, "cont",
                                                pool=pool)
            assert rel_l2(f(out), f(ref_out)) < TOL, f"call {it}"
        for i, s in enumerate(slots):
            r, c = pool.export(int(s), 0)
            assert rel_l2(r, rec[i]) < TOL
            assert np.array_equal(c, conv[i])


def test_chunked_prefill_strong_decay(gdn, synth, oracle):
    """Large A_log and a-gates: decays near underflow inside a chunk stay finite (log-space)."""
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    w = dict(w, A_log=np.full(cfg.hv, np.log(16.0), np.float32), dt_bias=np.full(cfg.hv, 3.0, np.float32))
    lens = [256]
    slots = np.array([0], np.int32)
    conv0, rec0 = synth.random_states(cfg, 1, seed=8, tag="decay")
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=1, device=0) as pool:
        pool.import_(0, 0, rec0[0], conv0[0])
        out, (ref_out, _, ref_rs, _) = _run(gdn, synth, oracle, cfg, w, lens, slots, conv0, rec0, 8, "decay",
                                            pool=pool)
        assert np.all(np.isfinite(f(out)))
        assert rel_l2(f(out), f(ref_out)) < TOL
        r, _ = pool.export(0, 0)
        assert np.all(np.isfinite(r))
        assert rel_l2(r, ref_rs[0]) < TOL


@pytest.mark.parametrize("pad", [0, 2])
def test_prep_forms_by_row_alignment(gdn, synth, oracle, pad):
    """The prep of a call with multi-token segments has an 8-channel form (16-byte aligned rows, pad 0) and a
    2-channel form (rows only 4-byte aligned, pad 2); both match the oracle, with decode tokens and segment
    starts inside the same 16-token tiles."""
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    lens = [1, 70, 2, 40, 1, 1, 100, 5]
    slots = np.array([3, 1, 6, 0, 5, 2, 4, 7], np.int32)
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=9, tag="pad")
    cu = _cu(lens)
    N = int(cu[-1])
    inp = synth.step_inputs(cfg, N, seed=9, tag="pad")

    def rows(a, ld):
        t = torch.zeros((N, ld), dtype=torch.bfloat16, device=DEV)
        t[:, :a.shape[1]] = gdn.bf16_to_device(a, DEV)
        return t[:, :a.shape[1]]

    qkv, z = rows(inp["qkv"], cfg.conv_dim + pad), rows(inp["z"], cfg.z_dim + pad)
    assert qkv.stride(0) == cfg.conv_dim + pad
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=8, device=0) as pool:
        pool.reserve_tokens(N)
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        out = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=DEV)
        pool.layer_step(0, gdn.LayerWeights(w, DEV), qkv, z, gdn.bf16_to_device(inp["ab"], DEV), out,
                        torch.from_numpy(slots).to(DEV), torch.from_numpy(cu).to(DEV), N)
        torch.cuda.synchronize()
        assert pool.check() == 0
        ref_out, ref_cs, ref_rs, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0, cu)
        got = gdn.bf16_to_host(out)
        for i, s in enumerate(slots):
            a, b = cu[i], cu[i + 1]
            assert rel_l2(f(got[a:b]), f(ref_out[a:b])) < TOL, f"output of segment {i} (T={lens[i]})"
            r, c = pool.export(int(s), 0)
            assert rel_l2(r, ref_rs[i]) < TOL, f"state of segment {i}"
            assert np.array_equal(c, ref_cs[i]), f"conv state of segment {i}"


def test_chunked_prefill_long_prompt_no_drift(gdn, synth, oracle):
    """A 4096-token prompt (64 chunks of the tensor-core path, each passing the f32 state through hi/lo bf16
    splits) packed with a decode token and a 700-token prompt, from random state: the last chunk's outputs and
    the final states are as close to the oracle as the first chunk's, so no error builds up over the chunks."""
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    lens = [4096, 1, 700]
    slots = np.array([2, 0, 5], np.int32)
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=12, tag="long")
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=8, device=0) as pool:
        pool.reserve_tokens(int(sum(lens)))
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        out, (ref_out, ref_cs, ref_rs, _) = _run(gdn, synth, oracle, cfg, w, lens, slots, conv0, rec0, 12, "long",
                                                 pool=pool)
        cu = _cu(lens)
        first = rel_l2(f(out[:64]), f(ref_out[:64]))
        last = rel_l2(f(out[4096 - 64:4096]), f(ref_out[4096 - 64:4096]))
        assert first < TOL and last < TOL, (first, last)
        for i, s in enumerate(slots):
            a, b = cu[i], cu[i + 1]
            assert rel_l2(f(out[a:b]), f(ref_out[a:b])) < TOL, f"output of segment {i} (T={lens[i]})"
            r, c = pool.export(int(s), 0)
            assert rel_l2(r, ref_rs[i]) < TOL, f"state of segment {i}"
            assert np.array_equal(c, ref_cs[i]), f"conv state of segment {i}"
