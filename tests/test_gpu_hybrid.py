"""GPU parity of the attention and MoE layer bodies (gdn_attn_step, gdn_moe_route, gdn_moe_step) against the
CPU restatement in oracle/hybrid_oracle.py, through the C ABI.

Tolerances: bf16 outputs whose inputs went through f32 (kernel) and f64 (oracle) accumulations of different
order, so single bf16 roundings may land one ulp apart; rel-L2 5e-3 on the roped K rows and the router
logits, 1e-2 on the attention and MoE outputs.  V rows are copied bit for bit.  Routing decisions are
compared on the kernel's own logits, so a one-ulp logit difference cannot flip an expert.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL_OUT = 1e-2
TOL_ROW = 5e-3


@pytest.fixture(scope="module")
def H():
    import __graft_entry__ as ge
    ge.load_oracle()
    return importlib.import_module("hybrid_oracle")


@pytest.fixture(scope="module")
def hy(pkg):
    return importlib.import_module("qwen_mlx_b200.hybrid")


def _bf16(synth, rng, shape, std=1.0):
    return synth.f32_to_bf16((rng.standard_normal(shape) * std).astype(np.float32))


def _attn_case(synth, cfg, n_slots, seed):
    rng = np.random.default_rng(seed)
    nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    caches = [_bf16(synth, rng, (n_slots, nkv, cfg.max_ctx, hd)) for _ in range(2)]   # garbage past every position
    gains = [synth.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)) for _ in range(2)]
    return rng, caches, gains


def _run_attn(synth, gdn, hy, H, cfg, slots, lens, positions, seed):
    dev = torch.device("cuda:0")
    n_slots = max(slots) + 2
    rng, (kc, vc), (qn, kn) = _attn_case(synth, cfg, n_slots, seed)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    qf = _bf16(synth, rng, (N, 2 * cfg.n_heads * cfg.head_dim))
    kin = _bf16(synth, rng, (N, cfg.n_kv_heads * cfg.head_dim))
    vin = _bf16(synth, rng, (N, cfg.n_kv_heads * cfg.head_dim))
    cache = hy.KVCache(cfg, n_slots, dev)
    cache.k.copy_(gdn.bf16_to_device(kc, dev).view(cache.k.shape))
    cache.v.copy_(gdn.bf16_to_device(vc, dev).view(cache.v.shape))
    b = lambda a: gdn.bf16_to_device(a, dev)  # noqa: E731
    out = hy.attn_step(cache, b(qf), b(kin), b(vin), b(qn), b(kn), slots, cu, positions)
    torch.cuda.synchronize()
    kc_o, vc_o = kc.copy(), vc.copy()
    ref = H.attn_step(cfg.as_dict(), qf, kin, vin, qn, kn, kc_o, vc_o, slots, cu, positions)
    got = gdn.bf16_to_host(out)
    kc_g = gdn.bf16_to_host(cache.k).reshape(kc.shape)
    vc_g = gdn.bf16_to_host(cache.v).reshape(vc.shape)
    return got, ref, (kc_g, vc_g), (kc_o, vc_o), cu


def _check_attn(H, got, ref, gpu_cache, orc_cache, slots, lens, positions):
    assert rel_l2(H.bf(got), H.bf(ref)) < TOL_OUT
    for s, n, p in zip(slots, lens, positions):
        if n == 0:
            continue
        kg, ko = gpu_cache[0][s, :, p:p + n], orc_cache[0][s, :, p:p + n]
        assert rel_l2(H.bf(kg), H.bf(ko)) < TOL_ROW
        assert np.array_equal(gpu_cache[1][s, :, p:p + n], orc_cache[1][s, :, p:p + n])
    # nothing outside the written rows changed
    mask = np.ones(gpu_cache[0].shape[:3], bool)
    for s, n, p in zip(slots, lens, positions):
        mask[s, :, p:p + n] = False
    assert np.array_equal(gpu_cache[1][mask], orc_cache[1][mask])
    assert np.array_equal(gpu_cache[0][mask], orc_cache[0][mask])


def test_attn_decode_qwen35_shapes(synth, gdn, hy, H):
    """Decode at the model's attention shapes (16 q heads, 2 kv heads, head_dim 256, rotary 64), contexts from
    1 key to most of the cache; split counts differ per token."""
    cfg = hy.AttnConfig(max_ctx=2048)
    slots, positions = [3, 0, 6, 1, 5, 2, 7, 4], [0, 1, 37, 255, 256, 900, 1500, 2047]
    lens = [1] * len(slots)
    got, ref, gc, oc, _ = _run_attn(synth, gdn, hy, H, cfg, slots, lens, positions, seed=1)
    _check_attn(H, got, ref, gc, oc, slots, lens, positions)


def test_attn_prefill_ragged(synth, gdn, hy, H):
    """Ragged prefill and continuation segments with one decode token, causal within each segment."""
    cfg = hy.AttnConfig(max_ctx=512)
    slots, lens, positions = [2, 0, 4, 1], [5, 1, 33, 70], [0, 12, 3, 200]
    got, ref, gc, oc, _ = _run_attn(synth, gdn, hy, H, cfg, slots, lens, positions, seed=2)
    _check_attn(H, got, ref, gc, oc, slots, lens, positions)


@pytest.mark.parametrize("hd,nh,nkv,rot", [(128, 8, 2, 32), (64, 4, 4, 64)])
def test_attn_other_head_dims(synth, gdn, hy, H, hd, nh, nkv, rot):
    cfg = hy.AttnConfig(n_heads=nh, n_kv_heads=nkv, head_dim=hd, rotary_dim=rot, rope_theta=10000.0, max_ctx=300)
    slots, lens, positions = [1, 0], [17, 1], [40, 299]
    got, ref, gc, oc, _ = _run_attn(synth, gdn, hy, H, cfg, slots, lens, positions, seed=3)
    _check_attn(H, got, ref, gc, oc, slots, lens, positions)


def test_attn_batch_invariance(synth, gdn, hy, H):
    """A sequence's output does not depend on what else is in the step (the reference's zero-padded batch
    does, mlx_executor.rs:57-86): decoding it alone and beside a long prefill gives identical bits."""
    cfg = hy.AttnConfig(max_ctx=1024)
    dev = torch.device("cuda:0")
    rng, (kc, vc), (qn, kn) = _attn_case(synth, cfg, 4, seed=4)
    b = lambda a: gdn.bf16_to_device(a, dev)  # noqa: E731
    D = cfg.n_heads * cfg.head_dim
    qf = _bf16(synth, rng, (301, 2 * D))
    kin = _bf16(synth, rng, (301, cfg.n_kv_heads * cfg.head_dim))
    vin = _bf16(synth, rng, (301, cfg.n_kv_heads * cfg.head_dim))

    def run(slots, cu, pos, rows):
        cache = hy.KVCache(cfg, 4, dev)
        cache.k.copy_(b(kc).view(cache.k.shape))
        cache.v.copy_(b(vc).view(cache.v.shape))
        out = hy.attn_step(cache, b(qf[rows]), b(kin[rows]), b(vin[rows]), b(qn), b(kn), slots, cu, pos)
        return gdn.bf16_to_host(out)

    alone = run([2], [0, 1], [40], [0])                                      # one key split
    mixed = run([2, 0, 1], [0, 1, 2, 52], [40, 900, 800], list(range(52)))  # four key splits
    assert np.array_equal(alone[0], mixed[0])


# ------------------------------------------------------------------ MoE

def _moe(synth, hy, cfg, seed):
    w = synth.moe_weights(cfg.hidden, cfg.n_experts, cfg.moe_inter, cfg.shared_inter, seed=seed)
    return w, hy.MoeWeights(w, torch.device("cuda:0"))


SMALL = dict(hidden=1024, n_experts=32, top_k=4, moe_inter=256, shared_inter=192, norm_topk_prob=True)


def _route_check(H, cfg, ids, wts, logits):
    oi, ow, p = H.moe_route(logits, cfg.top_k, cfg.norm_topk_prob)
    same = np.all(np.sort(ids, 1) == np.sort(oi, 1), axis=1)
    assert same.mean() >= 0.95
    for t in np.nonzero(~same)[0]:   # a differing pick is a near tie of probabilities
        kth = np.sort(p[t])[::-1][cfg.top_k - 1]
        for e in set(ids[t]) ^ set(oi[t]):
            assert abs(p[t, e] - kth) <= kth * 2.0 ** -7
    rows = np.nonzero(same)[0]
    # same experts; compare their weights expert by expert (near-equal probabilities may swap places)
    og, oo = np.argsort(ids[rows], 1), np.argsort(oi[rows], 1)
    wg = np.take_along_axis(wts[rows], og, 1)
    wo = np.take_along_axis(ow[rows], oo, 1)
    assert rel_l2(H.bf(wg), H.bf(wo)) < TOL_ROW


@pytest.mark.parametrize("norm", [True, False])
def test_moe_route(synth, gdn, hy, H, norm):
    cfg = hy.MoeConfig(**{**SMALL, "norm_topk_prob": norm})
    w, mw = _moe(synth, hy, cfg, seed=5)
    x = synth.normal_bf16(5, "moe.x", (64, cfg.hidden))
    ids, wts, logits = hy.moe_route(cfg, mw, gdn.bf16_to_device(x, torch.device("cuda:0")), want_logits=True)
    lg = gdn.bf16_to_host(logits)
    assert rel_l2(H.bf(lg), H.bf(H.moe_logits(x, w["router"]))) < TOL_ROW
    _route_check(H, cfg, ids.cpu().numpy(), gdn.bf16_to_host(wts), lg)


@pytest.mark.parametrize("n", [1, 8, 200])
def test_moe_step_small(synth, gdn, hy, H, n):
    """The whole block on the kernel's routing, against the oracle; 200 tokens put more pairs on the shared
    expert than one CTA's pair block holds."""
    cfg = hy.MoeConfig(**SMALL)
    w, mw = _moe(synth, hy, cfg, seed=6)
    x = synth.normal_bf16(6, f"moe.x{n}", (n, cfg.hidden))
    xd = gdn.bf16_to_device(x, torch.device("cuda:0"))
    ids, wts, _ = hy.moe_route(cfg, mw, xd)
    out_ext = hy.moe_step(cfg, mw, xd, route=(ids, wts))
    out_int = hy.moe_step(cfg, mw, xd)
    torch.cuda.synchronize()
    ref = H.moe_step(cfg.as_dict(), w, x, ids=ids.cpu().numpy(), weights=gdn.bf16_to_host(wts))
    got = gdn.bf16_to_host(out_ext)
    assert rel_l2(H.bf(got), H.bf(ref)) < TOL_OUT
    assert np.array_equal(got, gdn.bf16_to_host(out_int))   # the router inside the step gives the same bits


def test_moe_step_qwen35_shapes(synth, gdn, hy, H):
    """hidden 2048, top-8, expert and shared intermediate 512 (64 of the model's 256 experts, to keep the
    random checkpoint small)."""
    cfg = hy.MoeConfig(hidden=2048, n_experts=64, top_k=8, moe_inter=512, shared_inter=512)
    w, mw = _moe(synth, hy, cfg, seed=7)
    x = synth.normal_bf16(7, "moe.xq", (4, cfg.hidden))
    xd = gdn.bf16_to_device(x, torch.device("cuda:0"))
    ids, wts, logits = hy.moe_route(cfg, mw, xd, want_logits=True)
    out = hy.moe_step(cfg, mw, xd, route=(ids, wts))
    torch.cuda.synchronize()
    _route_check(H, cfg, ids.cpu().numpy(), gdn.bf16_to_host(wts), gdn.bf16_to_host(logits))
    ref = H.moe_step(cfg.as_dict(), w, x, ids=ids.cpu().numpy(), weights=gdn.bf16_to_host(wts))
    assert rel_l2(H.bf(gdn.bf16_to_host(out)), H.bf(ref)) < TOL_OUT
