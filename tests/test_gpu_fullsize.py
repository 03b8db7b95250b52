"""Parity at the reference model's full width against the committed full-size fixtures
(tests/golden/golden_full.npz, made by tests/golden/make_golden_full.py from the CPU oracle).

* The decode workload's own stack: 30 residual GDN layers with projections at hidden 2048,
  Hk 16 / Hv 32, 8 sequences, a 256-token prefill of each from zero state (one packed call per
  layer, the chunked tensor-core path), then 16 decode steps (qwen3_5.rs:559-669, :729-739).
  The tolerances were calibrated when the fixture was made: twice the distance between the
  oracle's default-order run and its runs with other valid GEMM accumulation orders (MLX matmul
  fixes none), floor 1e-3.
* The long-prompt prefill set at one layer: prompts of 512 ... 8192 tokens (30,016 tokens, up to
  128 chunks of 64 in one sequence), zero state, one packed call: the first rows and the last
  rows of every prompt (drift over the chunk chain), a strided sample of all outputs and of the
  final states within 1e-3, and the conv windows bit-exact.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_l2

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden_full as mgf  # noqa: E402

MANIFEST = json.loads((GOLDEN / "manifest_full.json").read_text())
SAMPLES = np.load(GOLDEN / "golden_full.npz")


def _s(name, key):
    return SAMPLES[f"{name}/{key}"]


@pytest.mark.gpu
def test_long_prompt_prefill_layer_matches_full_size_golden(gdn, synth):
    import torch
    dev = torch.device("cuda:0")
    meta = MANIFEST["cfg4_layer"]
    cfg, w, inp, cu = mgf.cfg4_inputs()
    n = len(cu) - 1
    N = int(cu[-1])
    slots = np.array([3, 9, 0, 14, 6, 11, 1, 8], np.int32)[:n]
    with gdn.StatePool(cfg, n_slots=16, device=0) as pool:
        pool.reserve_tokens(N)
        pool.reset(slots)
        lw = gdn.LayerWeights(w, dev)
        qkv = gdn.bf16_to_device(inp["qkv"], dev)
        z = gdn.bf16_to_device(inp["z"], dev)
        ab = gdn.bf16_to_device(inp["ab"], dev)
        out = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
        pool.layer_step(0, lw, qkv, z, ab, out, torch.from_numpy(slots).to(dev), torch.from_numpy(cu).to(dev), N)
        torch.cuda.synchronize()
        assert pool.check() == 0
        got_out = gdn.bf16_to_host(out)
        del qkv, z, ab, out
        states = [pool.export(int(s), 0) for s in slots]
    rs = np.stack([s[0] for s in states])
    cs = np.stack([s[1] for s in states])
    samples = mgf.cfg4_samples(got_out, rs, cu)
    f = synth.bf16_to_f32
    tol = meta["tolerance"]
    for i in range(n):
        for key in ("out_first4", "out_last8"):
            r = rel_l2(f(samples[key][i]), f(_s("cfg4_layer", key)[i]))
            assert r < tol[key], f"prompt {i} ({cfg4_len(meta, i)} tokens) {key}: rel-L2 {r:.2e}"
    assert rel_l2(f(samples["out_sample"]), f(_s("cfg4_layer", "out_sample"))) < tol["out_sample"]
    assert rel_l2(samples["rec_sample"], _s("cfg4_layer", "rec_sample")) < tol["rec_sample"]
    assert mgf.sha(cs) == meta["sha256"]["conv"], "conv windows differ from the oracle's"


def cfg4_len(meta, i):
    return meta["case"]["lens"][i]


@pytest.mark.gpu
def test_full_width_stack_prefill_then_decode_matches_full_size_golden(gdn, synth):
    import torch
    dev = torch.device("cuda:0")
    meta = MANIFEST["cfg2_stack"]
    case = meta["case"]
    B, P, n_dec = case["B"], case["prefill"], case["decode_steps"]
    cfg, ws, x_pre, x_dec, cu_pre = mgf.cfg2_inputs()
    L = cfg.n_layers
    slots = np.array([5, 2, 7, 0, 4, 9, 1, 6], np.int32)[:B]
    f = synth.bf16_to_f32
    tol = meta["tolerance"]
    with gdn.StatePool(cfg, n_slots=10, device=0) as pool:
        pool.reserve_tokens(B * P)
        mws = [gdn.MixerWeights(w, dev) for w in ws]
        del ws
        sl = torch.from_numpy(slots).to(dev)
        h = gdn.bf16_to_device(x_pre, dev)
        pool.stack_step(mws, h, sl, torch.from_numpy(cu_pre).to(dev), B * P)
        torch.cuda.synchronize()
        h_pre = gdn.bf16_to_host(h)
        cu_dec = torch.arange(B + 1, dtype=torch.int32, device=dev)
        outs = []
        for x in x_dec:
            hd = gdn.bf16_to_device(x, dev)
            pool.stack_step(mws, hd, sl, cu_dec, B)
            outs.append(hd)
        torch.cuda.synchronize()
        outs = [gdn.bf16_to_host(o) for o in outs]
        assert pool.check() == 0
        states = [[pool.export(int(s), l) for s in slots] for l in range(L)]
    rs = np.stack([[s[0] for s in row] for row in states])
    cs = np.stack([[s[1] for s in row] for row in states])
    got = mgf.cfg2_samples(h_pre, outs, cs, rs)
    r = rel_l2(f(got["prefill_last"]), f(_s("cfg2_stack", "prefill_last")))
    assert r < tol["prefill_last"], f"prefill last rows: rel-L2 {r:.2e} (tol {tol['prefill_last']:.2e})"
    r = rel_l2(f(got["prefill_sample"]), f(_s("cfg2_stack", "prefill_sample")))
    assert r < tol["prefill_sample"], f"prefill sample: rel-L2 {r:.2e}"
    ref_dec = _s("cfg2_stack", "decode_out")
    for s in range(n_dec):
        r = rel_l2(f(got["decode_out"][s]), f(ref_dec[s]))
        assert r < meta["decode_step_tolerance"][s], f"decode step {s}: rel-L2 {r:.2e}"
    assert rel_l2(f(got["decode_out"]), f(ref_dec)) < tol["decode_out"]
    r = rel_l2(got["rec_sample"], _s("cfg2_stack", "rec_sample"))
    assert r < tol["rec_sample"], f"recurrent states: rel-L2 {r:.2e}"
    r = rel_l2(f(got["conv_sample"]), f(_s("cfg2_stack", "conv_sample")))
    assert r < tol["conv_sample"], f"conv states: rel-L2 {r:.2e}"
