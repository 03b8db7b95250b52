"""gdn_layer_step_noalloc: the layer step for callers that cannot allocate device memory.

Such callers (an engine with a fixed device arena that forbids cudaMalloc after
start-up, or a framework whose caching allocator owns all device memory) keep
the states in their own buffers; the library brings a fixed, compiled-in
scratch array instead of allocating one.  The GPU test drives the new entry
point through the C ABI on caller-owned state and checks it against the pool
entry point gdn_layer_step on the same inputs, for two calls in a row (the
second call reuses the shared scratch the first one left behind).

This file is named to be collected last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

TOL = 1e-3   # the tolerance of the other parity tests (rel-L2, bf16 I/O, f32 state)


def _call(abi, cfg_c, n_slots, rec_ptr, conv_ptr, w_c, io_c, slot_ptr, cu_ptr, n_seq, n_tokens, stream):
    return abi.lib().gdn_layer_step_noalloc(C.byref(cfg_c), n_slots, rec_ptr, conv_ptr, C.byref(w_c), C.byref(io_c),
                                            slot_ptr, cu_ptr, n_seq, n_tokens, stream)


def test_noalloc_rejects_more_tokens_than_its_scratch(abi):
    """128 tokens fit at 32 v-heads; 129 are refused before any device work."""
    cfg = abi.GdnConfigC(2048, 16, 32, 128, 128, 4, 1, 1e-6)
    fake = C.c_void_p(1 << 20)   # aligned, never dereferenced: the size check comes first
    w = abi.GdnLayerWeightsC(fake.value, fake.value, fake.value, fake.value)
    io = abi.GdnStepIOC(fake.value, 8192, fake.value, 4096, fake.value, 64, fake.value, 4096)
    rc = _call(abi, cfg, 4, fake, fake, w, io, fake, fake, 1, 129, None)
    assert rc == abi.GDN_E_INVALID
    assert "scratch" in abi.last_error()


@pytest.mark.gpu
def test_noalloc_matches_pool_layer_step_two_calls(gdn, synth, abi):
    import torch

    dev = torch.device("cuda:0")
    cfg = synth.GdnConfig(n_layers=1)
    n_slots = 12
    lens = [1, 1, 3, 1, 2]                      # decode and short prefill segments in one packed call
    slots = np.array([7, 2, 10, 0, 5], np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    w = synth.layer_weights(cfg, 0, with_proj=False)
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=7, tag="noalloc")

    # caller-owned state for the no-alloc entry point: [n_slots][Hv][dv][dk] f32, [n_slots][K-1][D] bf16
    rec_t = torch.zeros((n_slots, cfg.hv, cfg.dv, cfg.dk), dtype=torch.float32, device=dev)
    conv_t = torch.zeros((n_slots, cfg.conv_k - 1, cfg.conv_dim), dtype=torch.bfloat16, device=dev)
    for i, s in enumerate(slots):
        rec_t[int(s)] = torch.from_numpy(rec0[i]).to(dev)
        conv_t[int(s)] = gdn.bf16_to_device(conv0[i], dev)

    lw = gdn.LayerWeights(w, dev)
    cfg_c = abi.GdnConfigC(cfg.hidden, cfg.hk, cfg.hv, cfg.dk, cfg.dv, cfg.conv_k, cfg.n_layers, cfg.eps)
    slots_d = torch.from_numpy(slots).to(dev)
    cu_d = torch.from_numpy(cu).to(dev)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    with gdn.StatePool(cfg, n_slots=n_slots, device=0) as pool:
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        for call in range(2):
            inp = synth.step_inputs(cfg, N, seed=100 + call, tag="noalloc")
            qkv = gdn.bf16_to_device(inp["qkv"], dev)
            z = gdn.bf16_to_device(inp["z"], dev)
            ab = gdn.bf16_to_device(inp["ab"], dev)
            out_ref = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
            out_new = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
            pool.layer_step(0, lw, qkv, z, ab, out_ref, slots_d, cu_d, N)
            io = abi.GdnStepIOC(qkv.data_ptr(), qkv.stride(0), z.data_ptr(), z.stride(0), ab.data_ptr(),
                                ab.stride(0), out_new.data_ptr(), out_new.stride(0))
            rc = _call(abi, cfg_c, n_slots, C.c_void_p(rec_t.data_ptr()), C.c_void_p(conv_t.data_ptr()), lw.c, io,
                       C.c_void_p(slots_d.data_ptr()), C.c_void_p(cu_d.data_ptr()), len(lens), N, stream)
            assert rc == abi.GDN_OK, abi.last_error()
            torch.cuda.synchronize()
            f = synth.bf16_to_f32
            assert rel_l2(f(gdn.bf16_to_host(out_new)), f(gdn.bf16_to_host(out_ref))) < TOL, f"call {call}: output"
            for s in slots:
                r_ref, c_ref = pool.export(int(s), 0)
                assert rel_l2(rec_t[int(s)].cpu().numpy(), r_ref) < TOL, f"call {call}: state of slot {s}"
                assert np.array_equal(gdn.bf16_to_host(conv_t[int(s)]), c_ref), f"call {call}: conv state of slot {s}"
