"""GPU parity of the stand-alone recurrence entry points against the oracle.

gdn_gated_delta_kernel (the reference-shaped drop-in for gated_delta_kernel,
metal_gdn.rs:170) and gdn_recurrence (pool-resident, ragged) are compared with
the CPU oracle on seeded inputs.  Tolerance: rel-L2 1e-3 on y and on the state
(bf16 I/O, f32 state); observed differences are f32 reassociation only.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _inputs(synth, B, T, hk, hv, seed=11, zero=False):
    q = synth.normal(seed, "gq", B * T * hk * 128).reshape(B, T, hk, 128)
    k = synth.normal(seed, "gk", B * T * hk * 128).reshape(B, T, hk, 128)
    q = synth.f32_to_bf16((q / np.sqrt((q * q).mean(-1, keepdims=True)) / 128).astype(np.float32))
    k = synth.f32_to_bf16((k / np.linalg.norm(k, axis=-1, keepdims=True)).astype(np.float32))
    v = synth.normal_bf16(seed, "gv", (B, T, hv, 128))
    g = synth.uniform(seed, "gg", B * T * hv, 0.3, 1.0).astype(np.float32).reshape(B, T, hv)
    beta = synth.f32_to_bf16(synth.uniform(seed, "gb", B * T * hv).astype(np.float32)).reshape(B, T, hv)
    st = np.zeros((B, hv, 128, 128), np.float32) if zero else \
        (synth.normal(seed, "gs", B * hv * 128 * 128) * 0.1).astype(np.float32).reshape(B, hv, 128, 128)
    return q, k, v, g, beta, st


def _dev(gdn, arrs, dev):
    q, k, v, g, beta, st = arrs
    b = gdn.bf16_to_device
    return b(q, dev), b(k, dev), b(v, dev), gdn.f32_to_device(g, dev), b(beta, dev), gdn.f32_to_device(st, dev)


@pytest.mark.parametrize("shape", [(1, 1, 16, 32), (8, 1, 16, 32), (1, 64, 16, 32), (3, 4, 2, 4), (2, 9, 1, 2),
                                   (2, 3, 4, 4)])
@pytest.mark.parametrize("inplace", [False, True])
def test_gated_delta_kernel_matches_oracle(gdn, synth, oracle, shape, inplace):
    B, T, hk, hv = shape
    dev = torch.device("cuda:0")
    arrs = _inputs(synth, B, T, hk, hv)
    q, k, v, g, beta, st = _dev(gdn, arrs, dev)
    if inplace:
        y, new = gdn.gated_delta_kernel(q, k, v, g, beta, st, T, B, hk, hv, 128, 128, out_state=st)
        assert new.data_ptr() == st.data_ptr()
    else:
        st0 = st.clone()
        y, new = gdn.gated_delta_kernel(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
        assert torch.equal(st, st0), "functional form must not modify the input state"
    torch.cuda.synchronize()
    y_ref, s_ref = oracle.recurrence(*arrs, T, B, hk, hv, 128, 128)
    f = synth.bf16_to_f32
    assert rel_l2(f(gdn.bf16_to_host(y)), f(y_ref)) < TOL
    assert rel_l2(new.cpu().numpy(), s_ref) < TOL


def test_gated_delta_kernel_matches_reference_golden(gdn, synth):
    """Against the committed outputs of the reference's own kernel body (config-1 shape, 64 tokens)."""
    import json
    import sys
    from pathlib import Path
    gdir = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(gdir))
    import make_golden as mg
    manifest = json.loads((gdir / "manifest.json").read_text())
    samples = np.load(gdir / "golden.npz")
    stride = manifest["sample_stride"]
    dev = torch.device("cuda:0")
    for case in mg.RECURRENCE_CASES:
        arrs = mg.recurrence_inputs(case)
        q, k, v, g, beta, st = _dev(gdn, arrs, dev)
        y, new = gdn.gated_delta_kernel(q, k, v, g, beta, st, case["T"], case["B"], case["hk"], case["hv"], 128, 128)
        torch.cuda.synchronize()
        f = synth.bf16_to_f32
        ys = gdn.bf16_to_host(y).reshape(-1)[::stride]
        ss = new.cpu().numpy().reshape(-1)[::stride]
        assert rel_l2(f(ys), f(samples[case["name"] + "/y"])) < TOL, case["name"]
        assert rel_l2(ss, samples[case["name"] + "/state"]) < TOL, case["name"]


def test_pool_recurrence_ragged_scrambled_slots(gdn, synth, oracle):
    """gdn_recurrence on pool slots: ragged lengths (incl. 0), scrambled slot ids, untouched slots unchanged."""
    cfg = synth.GdnConfig(n_layers=2)
    lens = [1, 5, 0, 2, 1, 9]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    slots = np.array([11, 3, 7, 0, 14, 6], np.int32)
    arrs = _inputs(synth, 1, N, cfg.hk, cfg.hv, seed=21)
    q, k, v, g, beta = (a[0] for a in arrs[:5])
    states = (synth.normal(21, "ps", len(lens) * cfg.hv * 128 * 128) * 0.1).astype(np.float32).reshape(
        len(lens), cfg.hv, 128, 128)
    dev = torch.device("cuda:0")
    with gdn.StatePool(cfg, n_slots=16, device=0) as pool:
        filler = (synth.normal(22, "fill", cfg.hv * 128 * 128)).astype(np.float32).reshape(cfg.hv, 128, 128)
        for s in range(16):
            pool.import_(s, 1, filler)
            pool.import_(s, 0, filler)
        for i, s in enumerate(slots):
            pool.import_(int(s), 1, states[i])
        b = gdn.bf16_to_device
        y = torch.zeros((N, cfg.hv, 128), dtype=torch.bfloat16, device=dev)
        pool.recurrence(1, b(q, dev), b(k, dev), b(v, dev), gdn.f32_to_device(g, dev), b(beta, dev), y,
                        torch.from_numpy(slots).to(dev), torch.from_numpy(cu).to(dev), N)
        torch.cuda.synchronize()
        assert pool.check() == 0
        y_ref, s_ref = oracle.recurrence_packed(q, k, v, g, beta, states, cu, cfg.hk, cfg.hv, 128, 128)
        f = synth.bf16_to_f32
        assert rel_l2(f(gdn.bf16_to_host(y)), f(y_ref)) < TOL
        for i, s in enumerate(slots):
            r, _ = pool.export(int(s), 1)
            if lens[i] == 0:
                assert np.array_equal(r, states[i])
            else:
                assert rel_l2(r, s_ref[i]) < TOL
        for s in range(16):                     # slots not in the batch, and the other layer: byte-identical
            if s not in slots:
                assert np.array_equal(pool.export(s, 1)[0], filler)
            assert np.array_equal(pool.export(s, 0)[0], filler)


def test_beta_g_kernel(gdn, synth, oracle):
    hv = 32
    ab = synth.normal_bf16(4, "bg", (37, 2 * hv))
    A_log = synth.uniform(4, "A", hv, 0.0, np.log(16.0)).astype(np.float32)
    dt = synth.uniform(4, "dt", hv, -1, 1).astype(np.float32)
    dev = torch.device("cuda:0")
    beta, g = gdn.beta_g(gdn.bf16_to_device(ab, dev), gdn.f32_to_device(A_log, dev), gdn.f32_to_device(dt, dev), hv)
    torch.cuda.synchronize()
    g_ref, beta_ref = oracle.gates(ab, A_log, dt, hv)
    assert rel_l2(g.cpu().numpy(), g_ref) < 1e-5
    mism = np.count_nonzero(gdn.bf16_to_host(beta) != beta_ref)
    assert mism <= 2   # bf16 rounding of sigmoid may flip only on ulp-level exp differences


def test_beta_g_kernel_bf16_dt_bias(gdn, synth, oracle):
    """gdn_beta_g_ex with a bf16 dt_bias: the add and its exp round to bf16, as in the oracle's bf16 mode."""
    hv = 32
    ab = synth.normal_bf16(5, "bg16", (41, 2 * hv))
    A_log = synth.uniform(5, "A", hv, 0.0, np.log(16.0)).astype(np.float32)
    dt = synth.bf16_to_f32(synth.f32_to_bf16(synth.uniform(5, "dt", hv, -1, 1).astype(np.float32)))
    dev = torch.device("cuda:0")
    beta, g = gdn.beta_g(gdn.bf16_to_device(ab, dev), gdn.f32_to_device(A_log, dev), gdn.f32_to_device(dt, dev), hv,
                         dt_bias_bf16=True)
    torch.cuda.synchronize()
    g_ref, beta_ref = oracle.gates(ab, A_log, dt, hv, dt_bias_bf16=True)
    g_f32, _ = oracle.gates(ab, A_log, dt, hv)
    assert rel_l2(g.cpu().numpy(), g_ref) < 1e-5
    assert rel_l2(g.cpu().numpy(), g_f32) > 1e-4        # the f32 gates are measurably different
    assert np.count_nonzero(gdn.bf16_to_host(beta) != beta_ref) <= 2

