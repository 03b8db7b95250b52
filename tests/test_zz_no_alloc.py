"""gdn_layer_step_noalloc: the layer step for callers that cannot allocate device memory.

Such callers (an engine with a fixed device arena that forbids cudaMalloc after
start-up, or a framework whose caching allocator owns all device memory) keep
the states in their own buffers; the library brings a fixed, compiled-in
scratch array instead of allocating one.  The GPU tests drive the new entry
point through the C ABI on caller-owned state, for two calls in a row (the
second call reuses the shared scratch the first one left behind), and check it
against the pool entry point gdn_layer_step on the same inputs -- the same
kernels, so outputs and states must be identical bit for bit -- and against the
CPU oracle within the parity tolerance.  The cases cover the two-kernel path
(mixed short segments), the fused decode kernel (64 and 128 one-token
sequences, the latter at the 4096-record limit) and a 128-token mixed call that
fills the array exactly.  gdn_noalloc_check reads the error word the kernels
write into the same array.

This file is named to be collected last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

TOL = 1e-3   # the tolerance of the other parity tests (rel-L2, bf16 I/O, f32 state), for the oracle comparison


def _call(abi, cfg_c, n_slots, rec_ptr, conv_ptr, w_c, io_c, slot_ptr, cu_ptr, n_seq, n_tokens, stream):
    return abi.lib().gdn_layer_step_noalloc(C.byref(cfg_c), n_slots, rec_ptr, conv_ptr, C.byref(w_c), C.byref(io_c),
                                            slot_ptr, cu_ptr, n_seq, n_tokens, stream)


def _flags(abi, reset=True) -> int:
    f = C.c_int32(-1)
    rc = abi.lib().gdn_noalloc_check(C.byref(f), 1 if reset else 0)
    assert rc == abi.GDN_OK, abi.last_error()
    return int(f.value)


def test_noalloc_rejects_more_tokens_than_its_scratch(abi):
    """128 tokens fit at 32 v-heads; 129 are refused before any device work."""
    cfg = abi.GdnConfigC(2048, 16, 32, 128, 128, 4, 1, 1e-6)
    fake = C.c_void_p(1 << 20)   # aligned, never dereferenced: the size check comes first
    w = abi.GdnLayerWeightsC(fake.value, fake.value, fake.value, fake.value, 0)
    io = abi.GdnStepIOC(fake.value, 8192, fake.value, 4096, fake.value, 64, fake.value, 4096)
    rc = _call(abi, cfg, 4, fake, fake, w, io, fake, fake, 1, 129, None)
    assert rc == abi.GDN_E_INVALID
    assert "scratch" in abi.last_error()


def test_noalloc_check_rejects_null(abi):
    assert abi.lib().gdn_noalloc_check(None, 0) == abi.GDN_E_INVALID


# (name, sequence lengths): a 128-token mixed call keeps every segment below 32 tokens, the length
# at which the pool entry point would switch those segments to the chunked tensor-core kernel.
_MIXED_128 = [31, 1, 30, 1, 1, 20, 1, 16, 1, 1, 12, 1, 2, 1, 5, 1, 1, 2]
CASES = [
    ("mixed_short", [1, 1, 3, 1, 2]),
    ("decode_64_fused", [1] * 64),
    ("decode_128_fused_at_limit", [1] * 128),
    ("mixed_128_at_limit", _MIXED_128),
]
assert sum(_MIXED_128) == 128


@pytest.mark.gpu
@pytest.mark.parametrize("name,lens", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_pool_layer_step_two_calls(gdn, synth, abi, oracle, name, lens):
    import torch

    dev = torch.device("cuda:0")
    cfg = synth.GdnConfig(n_layers=1)
    n = len(lens)
    n_slots = n + 7
    rng = np.random.default_rng(11)
    slots = rng.permutation(n_slots)[:n].astype(np.int32)   # scrambled, some slots left untouched
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    w = synth.layer_weights(cfg, 0, with_proj=False)
    conv0, rec0 = synth.random_states(cfg, n, seed=7, tag="noalloc" + name)

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
    f = synth.bf16_to_f32
    conv_ref, rec_ref = conv0, rec0                 # the oracle's running states, per sequence

    with gdn.StatePool(cfg, n_slots=n_slots, device=0) as pool:
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        for call in range(2):
            inp = synth.step_inputs(cfg, N, seed=100 + call, tag="noalloc" + name)
            qkv = gdn.bf16_to_device(inp["qkv"], dev)
            z = gdn.bf16_to_device(inp["z"], dev)
            ab = gdn.bf16_to_device(inp["ab"], dev)
            out_ref = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
            out_new = torch.empty((N, cfg.z_dim), dtype=torch.bfloat16, device=dev)
            pool.layer_step(0, lw, qkv, z, ab, out_ref, slots_d, cu_d, N)
            io = abi.GdnStepIOC(qkv.data_ptr(), qkv.stride(0), z.data_ptr(), z.stride(0), ab.data_ptr(),
                                ab.stride(0), out_new.data_ptr(), out_new.stride(0))
            rc = _call(abi, cfg_c, n_slots, C.c_void_p(rec_t.data_ptr()), C.c_void_p(conv_t.data_ptr()), lw.c, io,
                       C.c_void_p(slots_d.data_ptr()), C.c_void_p(cu_d.data_ptr()), n, N, stream)
            assert rc == abi.GDN_OK, abi.last_error()
            torch.cuda.synchronize()
            assert _flags(abi) == 0, f"call {call}: device error word set"
            assert pool.check() == 0
            got = gdn.bf16_to_host(out_new)
            # same kernels, same inputs: identical to the pool entry point
            assert np.array_equal(got, gdn.bf16_to_host(out_ref)), f"call {call}: output differs from gdn_layer_step"
            for s in slots:
                r_pool, c_pool = pool.export(int(s), 0)
                assert np.array_equal(rec_t[int(s)].cpu().numpy(), r_pool), f"call {call}: state of slot {s}"
                assert np.array_equal(gdn.bf16_to_host(conv_t[int(s)]), c_pool), f"call {call}: conv of slot {s}"
            # and within the parity tolerance of the CPU oracle
            o_ref, conv_ref, rec_ref, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv_ref,
                                                            rec_ref, cu)
            assert rel_l2(f(got), f(o_ref)) < TOL, f"call {call}: output vs oracle"
            rec_all = np.stack([rec_t[int(s)].cpu().numpy() for s in slots])
            assert rel_l2(rec_all, rec_ref) < TOL, f"call {call}: states vs oracle"
            conv_all = np.stack([gdn.bf16_to_host(conv_t[int(s)]) for s in slots])
            assert np.array_equal(conv_all, conv_ref), f"call {call}: conv states vs oracle"
        # slots no sequence used stay zero
        used = set(int(s) for s in slots)
        for s in range(n_slots):
            if s not in used:
                assert not rec_t[s].any() and not conv_t[s].any()


@pytest.mark.gpu
def test_noalloc_check_reports_a_skipped_bad_slot(gdn, synth, abi, oracle):
    """A slot id outside [0, n_slots) in the device table: the kernels skip that sequence and set
    1 << GDN_E_BAD_SLOT in the no-alloc error word; gdn_noalloc_check reports and clears it, and the
    good sequence of the same call is still correct."""
    import torch

    dev = torch.device("cuda:0")
    cfg = synth.GdnConfig(n_layers=1)
    n_slots = 4
    slots = np.array([2, 40], np.int32)     # 40 is out of range: rejected by the kernels' own checks
    cu = np.array([0, 1, 2], np.int32)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    conv0, rec0 = synth.random_states(cfg, 1, seed=9, tag="noalloc_bad")
    inp = synth.step_inputs(cfg, 2, seed=9, tag="noalloc_bad")
    rec_t = torch.zeros((n_slots, cfg.hv, cfg.dv, cfg.dk), dtype=torch.float32, device=dev)
    conv_t = torch.zeros((n_slots, cfg.conv_k - 1, cfg.conv_dim), dtype=torch.bfloat16, device=dev)
    rec_t[2] = torch.from_numpy(rec0[0]).to(dev)
    conv_t[2] = gdn.bf16_to_device(conv0[0], dev)
    lw = gdn.LayerWeights(w, dev)
    cfg_c = abi.GdnConfigC(cfg.hidden, cfg.hk, cfg.hv, cfg.dk, cfg.dv, cfg.conv_k, cfg.n_layers, cfg.eps)
    qkv = gdn.bf16_to_device(inp["qkv"], dev)
    z = gdn.bf16_to_device(inp["z"], dev)
    ab = gdn.bf16_to_device(inp["ab"], dev)
    out = torch.zeros((2, cfg.z_dim), dtype=torch.bfloat16, device=dev)
    io = abi.GdnStepIOC(qkv.data_ptr(), qkv.stride(0), z.data_ptr(), z.stride(0), ab.data_ptr(), ab.stride(0),
                        out.data_ptr(), out.stride(0))
    slots_d = torch.from_numpy(slots).to(dev)
    cu_d = torch.from_numpy(cu).to(dev)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _flags(abi)                                 # start from a clear word
    rc = _call(abi, cfg_c, n_slots, C.c_void_p(rec_t.data_ptr()), C.c_void_p(conv_t.data_ptr()), lw.c, io,
               C.c_void_p(slots_d.data_ptr()), C.c_void_p(cu_d.data_ptr()), 2, 2, stream)
    assert rc == abi.GDN_OK, abi.last_error()
    flags = _flags(abi, reset=False)
    assert flags & (1 << abi.GDN_E_BAD_SLOT)
    assert _flags(abi) == flags                 # read again, then cleared
    assert _flags(abi) == 0
    ref = oracle.layer_step(cfg, w, inp["qkv"][:1], inp["z"][:1], inp["ab"][:1], conv0, rec0, cu[:2])
    f = synth.bf16_to_f32
    assert rel_l2(f(gdn.bf16_to_host(out[:1])), f(ref[0])) < TOL
    for s in (0, 1, 3):
        assert not rec_t[s].any() and not conv_t[s].any()
