"""CPU tests of the attention / MoE layer bodies: the oracle's own properties and pins, and the C ABI's host-side
argument checks (no GPU work is issued: every call here fails its checks before touching the device)."""
from __future__ import annotations

import ctypes as C
import importlib

import numpy as np
import pytest


@pytest.fixture(scope="module")
def H():
    import __graft_entry__ as ge
    ge.load_oracle()
    return importlib.import_module("hybrid_oracle")


@pytest.fixture(scope="module")
def hy(pkg):
    return importlib.import_module("qwen_mlx_b200.hybrid")


# ------------------------------------------------------------------ oracle pins and properties

def test_q4_dequant_matches_projection_oracle(H, synth, oracle):
    """The experts' dequantisation is the projections' (gdn_oracle.q4_dequantize), bit for bit."""
    m = synth.q4_matrix(3, "pin", 128, 512)
    assert np.array_equal(H.q4_dequant(m, slice(0, 128)), oracle.q4_dequantize(m["q"], m["scales"], m["biases"]))


def test_rope_depends_on_relative_position(H):
    """<rope(q, m), rope(k, n)> depends on m - n only (up to the bf16 rounding of the rotated vectors)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal(256).astype(np.float32)
    k = rng.standard_normal(256).astype(np.float32)
    dots = [float(H.rope(q[None], np.array([m]), 64, 1e7)[0] @ H.rope(k[None], np.array([m - 7]), 64, 1e7)[0])
            for m in (7, 100, 1000, 4000)]
    assert np.ptp(dots) < 2e-2 * abs(dots[0]) + 0.05
    # dims past rotary_dim are untouched (only rounded)
    r = H.rope(q[None], np.array([123]), 64, 1e7)[0]
    assert np.array_equal(r[64:], H.rbf(q[64:]))


def test_attn_oracle_masks_other_keys(H, synth):
    """A token's output ignores cache rows past its position and every other slot's rows."""
    cfg = dict(n_heads=4, n_kv_heads=2, head_dim=64, rotary_dim=16, rope_theta=1e4, rms_norm_eps=1e-6)
    rng = np.random.default_rng(1)
    bfr = lambda shape: synth.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))  # noqa: E731
    qf, kin, vin = bfr((3, 4 * 128)), bfr((3, 2 * 64)), bfr((3, 2 * 64))
    qn = kn = synth.f32_to_bf16(np.ones(64, np.float32))
    kc, vc = bfr((2, 2, 32, 64)), bfr((2, 2, 32, 64))
    out1 = H.attn_step(cfg, qf, kin, vin, qn, kn, kc.copy(), vc.copy(), [1], [0, 3], [5])
    kc2, vc2 = kc.copy(), vc.copy()
    kc2[1, :, 8:] = bfr((2, 24, 64))   # rows past the last token's position (7)
    vc2[1, :, 8:] = bfr((2, 24, 64))
    kc2[0], vc2[0] = bfr((2, 32, 64)), bfr((2, 32, 64))
    out2 = H.attn_step(cfg, qf, kin, vin, qn, kn, kc2, vc2, [1], [0, 3], [5])
    assert np.array_equal(out1, out2)


def test_moe_route_ties_and_renormalisation(H, synth):
    logits = synth.f32_to_bf16(np.array([[1.0, 3.0, 3.0, 2.0, 3.0, -1.0]], np.float32))
    ids, w, p = H.moe_route(logits, 3, True)
    assert ids.tolist() == [[1, 2, 4]]   # equal probabilities: lower index first
    assert abs(float(H.bf(w).sum()) - 1.0) < 1e-2
    ids2, w2, _ = H.moe_route(logits, 3, False)
    assert np.array_equal(H.bf(w2), p[0, [1, 2, 4]][None])


# ------------------------------------------------------------------ ABI host checks

def _acfg(hy, **kw):
    return hy.AttnConfig(**kw).c()


def test_attn_workspace_query(abi, hy):
    L = abi.lib()
    out = C.c_int64(0)
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy)), 8, 4096, C.byref(out)) == abi.GDN_OK
    # 8 decode tokens, 16 heads of 256: per-(token, head) partials of up to 16 key splits dominate
    assert out.value >= 8 * 16 * 16 * 256 * 4
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, head_dim=96)), 8, 64, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, n_heads=6, n_kv_heads=4)), 8, 64, C.byref(out)) == \
        abi.GDN_E_INVALID
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, rotary_dim=63)), 8, 64, C.byref(out)) == abi.GDN_E_INVALID


@pytest.mark.parametrize("slots,lens,positions,code", [
    ([1, 1], [1, 1], [0, 0], 3),        # slot used twice
    ([4], [1], [0], 3),                 # slot out of range (4 slots)
    ([0, 1], [1, 2], [0, 15], 1),       # position + tokens past max_ctx (16)
    ([0], [1], [-1], 1),                # negative position
])
def test_attn_step_rejects_bad_tables(abi, hy, slots, lens, positions, code):
    cfg = _acfg(hy, max_ctx=16)
    s = np.asarray(slots, np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    pos = np.asarray(positions, np.int32)
    fake = C.c_void_p(256)   # device pointers are never touched on a failing call
    rc = abi.lib().gdn_attn_step(C.byref(cfg), fake, fake, fake, fake, fake, fake, fake, 4,
                                 s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                                 pos.ctypes.data_as(C.c_void_p), len(s), int(cu[-1]), fake, fake, 1 << 30, None)
    assert rc == code, abi.last_error()
    assert abi.last_error()


def test_attn_step_bad_seqlens(abi, hy):
    cfg = _acfg(hy, max_ctx=16)
    s = np.asarray([0, 1], np.int32)
    cu = np.asarray([0, 2, 1], np.int32)
    pos = np.zeros(2, np.int32)
    fake = C.c_void_p(256)
    rc = abi.lib().gdn_attn_step(C.byref(cfg), fake, fake, fake, fake, fake, fake, fake, 4,
                                 s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                                 pos.ctypes.data_as(C.c_void_p), 2, 1, fake, fake, 1 << 30, None)
    assert rc == abi.GDN_E_BAD_SEQLENS


def test_moe_workspace_and_checks(abi, hy):
    L = abi.lib()
    out = C.c_int64(0)
    cfg = hy.MoeConfig()
    assert L.gdn_moe_workspace_bytes(C.byref(cfg.c()), 8, C.byref(out)) == abi.GDN_OK
    assert out.value >= 8 * 9 * (512 + 2048) * 2   # h and y rows of every (token, expert) pair
    bad = hy.MoeConfig(hidden=2000).c()
    assert L.gdn_moe_workspace_bytes(C.byref(bad), 8, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    bad = hy.MoeConfig(top_k=17).c()
    assert L.gdn_moe_workspace_bytes(C.byref(bad), 8, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    # routing given half-way: rejected before any launch
    fake = C.c_void_p(256)
    q = abi.GdnQ4MatrixC(fake, fake, fake)
    w = abi.GdnMoeWeightsC(fake, q, q, q, q, q, q, fake)
    rc = L.gdn_moe_step(C.byref(cfg.c()), C.byref(w), fake, 4, fake, None, fake, fake, 1 << 30, None)
    assert rc == abi.GDN_E_INVALID
    rc = L.gdn_moe_step(C.byref(cfg.c()), C.byref(w), fake, 4, None, None, fake, fake, 16, None)
    assert rc == abi.GDN_E_INVALID and "workspace" in abi.last_error()
