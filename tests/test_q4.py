"""CPU checks of the 4-bit weight format used by the quantized projections: the synthetic quantizer
(affine, groups of 64 columns, MLX's bit packing) and the oracle's dequantization / quantized linear."""
from __future__ import annotations

import numpy as np


def test_quantizer_packs_mlx_layout_and_bounds_the_error(synth, oracle):
    w = synth.normal_bf16(1, "q4cpu", (96, 256), 0.02)
    w_q, s, b = synth.quantize_q4(w)
    assert w_q.dtype == np.uint32 and w_q.shape == (96, 32)
    assert s.shape == b.shape == (96, 4)
    f = synth.bf16_to_f32
    # column k sits in bits 4*(k%8) of word k/8
    k = 77
    q = (w_q[:, k // 8] >> np.uint32(4 * (k % 8))) & np.uint32(0xF)
    manual = f(synth.f32_to_bf16((f(s[:, k // 64]) * q + f(b[:, k // 64])).astype(np.float32)))
    deq = f(oracle.q4_dequantize(w_q, s, b))
    assert np.allclose(deq[:, k], manual, rtol=2 ** -7, atol=0)
    # error within half a step (plus the bf16 rounding of the dequantized weight)
    err = np.abs(deq - f(w)).reshape(96, 4, 64).max(axis=2)
    assert np.all(err <= 0.5 * f(s) * 1.05 + 2 ** -8 * np.abs(f(w)).reshape(96, 4, 64).max(axis=2))


def test_dequantize_rounds_once(synth, oracle):
    # scale * q + bias exact in f64, then one round-to-nearest-even to bf16
    w_q = np.array([[0xFEDCBA98]], np.uint32).repeat(8, axis=1)            # one row, 64 columns
    s = synth.f32_to_bf16(np.array([[0.0078125 * 1.0078125]], np.float32))
    b = synth.f32_to_bf16(np.array([[-0.0625]], np.float32))
    d = synth.bf16_to_f32(oracle.q4_dequantize(w_q, s, b))[0]
    sv, bv = synth.bf16_to_f32(s)[0, 0], synth.bf16_to_f32(b)[0, 0]
    for col, code in enumerate([8, 9, 10, 11, 12, 13, 14, 15]):
        exact = np.float64(sv) * code + np.float64(bv)
        cand = synth.bf16_to_f32(synth.f32_to_bf16(np.array([exact], np.float32)))[0]
        assert abs(d[col] - exact) <= abs(cand - exact) + 1e-12


def test_q4_linear_matches_linear_on_dequantized(synth, oracle):
    w = synth.normal_bf16(2, "q4lin", (64, 128), 0.02)
    x = synth.normal_bf16(3, "q4lin_x", (5, 128))
    q = synth.quantize_q4(w)
    assert np.array_equal(oracle.q4_linear(x, *q), oracle.linear(x, oracle.q4_dequantize(*q)))
