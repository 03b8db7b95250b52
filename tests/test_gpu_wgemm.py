"""GPU parity of the weight-streaming projection kernel: bf16 tiles (gdn_weight_tile +
gdn_linear_tiled) and MLX 4-bit tiles (gdn_weight_tile_q4 + gdn_linear_q4, the reference's
quantized projections).

* Both tiled layouts are compared byte for byte with numpy restatements.
* y = x w^T against the exact f64 product of x and the (dequantized) bf16 weight: every output
  within one bf16 ulp plus the f32 dot-product error bound 2^-16 * sum|x*w|, and more than 99% of
  outputs exactly the correctly rounded value (the bar the cuBLASLt path meets), over the Qwen3.5
  projection shapes (in-projection 12352 x 2048, out-projection 2048 x 4096) and ragged ones, with
  each token padding (16/32/64), token blocks beyond 64, and strided x / y.
* The stream-K sum order is fixed: repeated runs agree bit for bit.
* A whole mixer layer on 4-bit weights agrees with the oracle on the dequantized weights (the
  tolerance calibrated on the oracle's own accumulation-order spread, as in test_gpu_mixer.py), and
  a mixer layer on bf16 tiles agrees with the same layer on cuBLASLt."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ALT_ORDERS, order_noise, rel_l2, with_order

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = 1e-3


def _tile_ref(w: np.ndarray) -> np.ndarray:
    """bf16 block (kt, rg) = rows [8 rg, +8) x columns [64 kt, +64) in 1 KB at (kt * NRG + rg) * 1024,
    element (8 rg + r, 64 kt + 8 c + e) at byte c*128 + r*16 + e*2, zero padded."""
    N, K = w.shape
    NRG, KT = -(-N // 8), -(-K // 64)
    wp = np.zeros((NRG * 8, KT * 64), np.uint16)
    wp[:N, :K] = w
    # [rg][r][kt][c][e] -> [kt][rg][c][r][e]
    return np.ascontiguousarray(wp.reshape(NRG, 8, KT, 8, 8).transpose(2, 0, 3, 1, 4)).reshape(-1).view(np.uint8)


def _tile_q4_ref(w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray) -> np.ndarray:
    """4-bit block (kt, rg) in 288 B at (kt * NRG + rg) * 288: word (c, r) at c*32 + r*4 with the codes of
    columns 64 kt + 8c .. +7 of row 8 rg + r (column 8c+e in nibble e/2, e even, or 4 + e/2, e odd),
    scales at 256, biases at 272."""
    N, K8 = w_q.shape
    K = K8 * 8
    NRG, KT = -(-N // 8), K // 64
    shifts = np.arange(8, dtype=np.uint32) * 4
    codes = (w_q[:, :, None] >> shifts) & np.uint32(0xF)                      # [N][K/8][e]
    pos = np.array([0, 4, 1, 5, 2, 6, 3, 7])                                 # nibble of column e
    words = np.zeros((NRG * 8, K8), np.uint32)
    for e in range(8):
        words[:N] |= codes[:, :, e] << np.uint32(4 * pos[e])
    sp = np.zeros((NRG * 8, KT), np.uint16)
    bp = np.zeros((NRG * 8, KT), np.uint16)
    sp[:N], bp[:N] = scales, biases
    out = np.zeros((KT, NRG, 288), np.uint8)
    w4 = words.reshape(NRG, 8, KT, 8).transpose(2, 0, 3, 1)                  # [kt][rg][c][r]
    out[:, :, :256] = np.ascontiguousarray(w4).reshape(KT, NRG, -1).view(np.uint8)
    out[:, :, 256:272] = np.ascontiguousarray(sp.reshape(NRG, 8, KT).transpose(2, 0, 1)).view(np.uint8)
    out[:, :, 272:] = np.ascontiguousarray(bp.reshape(NRG, 8, KT).transpose(2, 0, 1)).view(np.uint8)
    return out.reshape(-1)


def _check_exact(synth, x, w, got):
    f = synth.bf16_to_f32
    xf, wf = f(x).astype(np.float64), f(w).astype(np.float64)
    exact = xf @ wf.T
    got = f(got).astype(np.float64)
    rounded = f(synth.f32_to_bf16(exact.astype(np.float32))).astype(np.float64)
    ulp = np.ldexp(1.0, np.frexp(np.abs(exact))[1] - 8)
    bound = ulp + 2.0 ** -16 * (np.abs(xf) @ np.abs(wf).T)
    assert np.all(np.abs(got - exact) <= bound)
    assert (got == rounded).mean() > 0.99


@pytest.mark.parametrize("shape", [(300, 200), (12352, 2048), (129, 72)])
def test_tiled_layout_matches_restatement(gdn, synth, shape):
    w = synth.normal_bf16(5, f"tile{shape}", shape)
    t = gdn.tile_weight(gdn.bf16_to_device(w, DEV))
    torch.cuda.synchronize()
    assert np.array_equal(t.cpu().numpy(), _tile_ref(w))


@pytest.mark.parametrize("shape", [(300, 192), (2048, 4096)])
def test_q4_tiled_layout_matches_restatement(gdn, synth, shape):
    w_q, s, b = synth.quantize_q4(synth.normal_bf16(5, f"q4tile{shape}", shape, 0.02))
    t = gdn.q4_to_device(w_q, s, b, DEV)
    torch.cuda.synchronize()
    assert np.array_equal(t.cpu().numpy(), _tile_q4_ref(w_q, s, b))


CASES = [
    ((12352, 2048), (1, 8, 16, 17, 64)),
    ((2048, 4096), (3, 8, 33)),
    ((300, 192), (5, 32, 64, 70)),
    ((129, 128), (2, 130)),
]


def _run(gdn, pool, q4, tiles, x, N, K, M):
    xd = torch.zeros((M, K + 8), dtype=torch.bfloat16, device=DEV)     # strided x (ld K + 8)
    xd[:, :K] = gdn.bf16_to_device(x, DEV)
    yd = torch.full((M, N + 3), 7.0, dtype=torch.bfloat16, device=DEV)  # strided y (ld N + 3)
    if q4:
        pool.linear_q4(xd[:, :K], tiles, N, yd[:, :N])
    else:
        pool.linear_tiled(xd[:, :K], tiles, N, yd[:, :N])
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert torch.all(yd[:, N:] == 7.0), "wrote past n_out"
    return gdn.bf16_to_host(yd[:, :N].contiguous())


@pytest.mark.parametrize("shape,ms", CASES)
def test_linear_tiled_within_one_ulp_of_exact(gdn, synth, shape, ms):
    cfg = synth.GdnConfig(n_layers=1)
    N, K = shape
    w = synth.normal_bf16(6, f"lt{shape}", shape)
    with gdn.StatePool(cfg, n_slots=1, device=0) as pool:
        wt = gdn.tile_weight(gdn.bf16_to_device(w, DEV))
        for M in ms:
            x = synth.normal_bf16(7, f"ltx{shape}{M}", (M, K))
            _check_exact(synth, x, w, _run(gdn, pool, False, wt, x, N, K, M))


@pytest.mark.parametrize("shape,ms", CASES)
def test_linear_q4_within_one_ulp_of_exact(gdn, synth, oracle, shape, ms):
    cfg = synth.GdnConfig(n_layers=1)
    N, K = shape
    w_q, s, b = synth.quantize_q4(synth.normal_bf16(6, f"q4{shape}", shape, 0.02))
    w_deq = oracle.q4_dequantize(w_q, s, b)
    with gdn.StatePool(cfg, n_slots=1, device=0) as pool:
        wt = gdn.q4_to_device(w_q, s, b, DEV)
        for M in ms:
            x = synth.normal_bf16(7, f"q4x{shape}{M}", (M, K))
            _check_exact(synth, x, w_deq, _run(gdn, pool, True, wt, x, N, K, M))


@pytest.mark.parametrize("q4", [False, True])
def test_linear_repeats_bit_for_bit(gdn, synth, q4):
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.normal_bf16(9, "rep_w", (2048, 4096), 0.02)
    x = gdn.bf16_to_device(synth.normal_bf16(9, "rep_x", (8, 4096)), DEV)
    with gdn.StatePool(cfg, n_slots=1, device=0) as pool:
        wt = gdn.q4_to_device(*synth.quantize_q4(w), DEV) if q4 else gdn.tile_weight(gdn.bf16_to_device(w, DEV))
        ys = []
        for _ in range(3):
            y = torch.empty((8, 2048), dtype=torch.bfloat16, device=DEV)
            (pool.linear_q4 if q4 else pool.linear_tiled)(x, wt, 2048, y)
            ys.append(y)
        torch.cuda.synchronize()
        assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


def test_linear_tiled_rejects_unaligned_rows(gdn, synth, abi):
    cfg = synth.GdnConfig(n_layers=1)
    with gdn.StatePool(cfg, n_slots=1, device=0) as pool:
        wt = gdn.tile_weight(torch.zeros((256, 128), dtype=torch.bfloat16, device=DEV))
        x = torch.zeros((4, 133), dtype=torch.bfloat16, device=DEV)
        y = torch.zeros((4, 256), dtype=torch.bfloat16, device=DEV)
        with pytest.raises(abi.GdnError) as e:
            pool.linear_tiled(x[:, :128], wt, 256, y)  # ld_x = 133: rows not 16-byte aligned
        assert e.value.code == abi.GDN_E_INVALID


def _q4_mixer_weights(synth, oracle, w):
    """4-bit in/out projections of a synthetic layer, and the weight dict the oracle runs: the same
    layer with each projection replaced by its dequantized bf16 value."""
    w_in = np.concatenate([w["w_qkv"], w["w_z"], w["w_b"], w["w_a"]], axis=0)
    q_in, q_out = synth.quantize_q4(w_in), synth.quantize_q4(w["w_out"])
    d_in = oracle.q4_dequantize(*q_in)
    wd = dict(w)
    D, Z, hv = w["w_qkv"].shape[0], w["w_z"].shape[0], w["w_b"].shape[0]
    wd["w_qkv"], wd["w_z"] = d_in[:D], d_in[D:D + Z]
    wd["w_b"], wd["w_a"] = d_in[D + Z:D + Z + hv], d_in[D + Z + hv:]
    wd["w_out"] = oracle.q4_dequantize(*q_out)
    return (q_in, q_out), wd


@pytest.mark.parametrize("lens", [[1] * 8, [1, 3, 1, 6, 0, 2], [70, 1]])
def test_mixer_step_q4_matches_oracle(gdn, synth, oracle, lens):
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=True)
    q4, wd = _q4_mixer_weights(synth, oracle, w)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    slots = np.arange(len(lens), dtype=np.int32)[::-1].copy()
    x = synth.normal_bf16(3, "q4mix_x", (N, cfg.hidden))
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=5, tag="q4mix")
    with gdn.StatePool(cfg, n_slots=len(lens), device=0) as pool:
        for i, s in enumerate(slots):
            pool.import_(int(s), 0, rec0[i], conv0[i])
        mw = gdn.MixerWeights(w, DEV, q4=q4)
        y = torch.empty((N, cfg.hidden), dtype=torch.bfloat16, device=DEV)
        pool.mixer_step(0, mw, gdn.bf16_to_device(x, DEV), y, torch.from_numpy(slots).to(DEV),
                        torch.from_numpy(cu).to(DEV), N)
        torch.cuda.synchronize()
        assert pool.check() == 0
        got_rec = np.stack([pool.export(int(slots[i]), 0)[0] for i in range(len(lens)) if lens[i] > 0])
    y_ref, _, rs_ref = oracle.mixer_step(cfg, wd, x, conv0, rec0, cu)
    alts = [with_order(oracle, o, lambda: oracle.mixer_step(cfg, wd, x, conv0, rec0, cu)) for o in ALT_ORDERS]
    f = synth.bf16_to_f32
    tol = max(TOL, 2 * order_noise(y_ref, [a[0] for a in alts], f))
    assert rel_l2(f(gdn.bf16_to_host(y)), f(y_ref)) < tol
    keep = [i for i in range(len(lens)) if lens[i] > 0]
    assert rel_l2(got_rec, rs_ref[keep]) < max(TOL, 2 * order_noise(rs_ref[keep], [a[2][keep] for a in alts]))


def test_mixer_step_bf16_tiles_match_cublaslt(gdn, synth):
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=True)
    lens = [1, 3, 1, 6, 0, 2]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    slots = np.arange(len(lens), dtype=np.int32)
    x = gdn.bf16_to_device(synth.normal_bf16(3, "mt_x", (N, cfg.hidden)), DEV)
    conv0, rec0 = synth.random_states(cfg, len(lens), seed=4, tag="mt")
    outs = []
    for tiled in (True, False):
        with gdn.StatePool(cfg, n_slots=len(lens), device=0) as pool:
            for i, s in enumerate(slots):
                pool.import_(int(s), 0, rec0[i], conv0[i])
            mw = gdn.MixerWeights(w, DEV, tiled=tiled)
            y = torch.empty((N, cfg.hidden), dtype=torch.bfloat16, device=DEV)
            pool.mixer_step(0, mw, x, y, torch.from_numpy(slots).to(DEV), torch.from_numpy(cu).to(DEV), N)
            torch.cuda.synchronize()
            assert pool.check() == 0
            outs.append(synth.bf16_to_f32(gdn.bf16_to_host(y)))
    # both round the same f32 products to bf16; a flipped rounding in a projection output moves the
    # layer's output by up to ~1e-3 (the calibrated mixer tolerance of test_gpu_mixer.py)
    assert rel_l2(outs[0], outs[1]) < 3e-3
