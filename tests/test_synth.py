"""CPU tests of the seeded synthetic generator and the bf16 helpers."""
from __future__ import annotations

import numpy as np


def test_generator_is_deterministic_and_stream_separated(synth):
    a = synth.normal(0, "x", 1000)
    b = synth.normal(0, "x", 1000)
    c = synth.normal(0, "y", 1000)
    d = synth.normal(1, "x", 1000)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c) and not np.array_equal(a, d)
    # prefix property: the first n values do not depend on how many are drawn
    assert np.array_equal(synth.normal(0, "x", 10), a[:10])


def test_generator_moments(synth):
    x = synth.normal(0, "m", 200_000)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    u = synth.uniform(0, "u", 200_000, -1, 1)
    assert u.min() >= -1 and u.max() < 1 and abs(u.mean()) < 0.01


def test_bf16_round_trip_and_rne(synth):
    x = np.array([1.0, -2.5, 3.140625, 0.0, 65536.0], np.float32)   # all exactly representable
    assert np.array_equal(synth.bf16_to_f32(synth.f32_to_bf16(x)), x)
    # ties go to even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7
    t = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8], np.float32)
    assert np.array_equal(synth.bf16_to_f32(synth.f32_to_bf16(t)), np.array([1.0, 1.0 + 2.0 ** -6], np.float32))


def test_layer_weight_shapes(synth):
    cfg = synth.QWEN35_35B_A3B
    w = synth.layer_weights(cfg, 3, with_proj=True)
    assert cfg.conv_dim == 8192 and cfg.z_dim == 4096
    assert w["conv_w"].shape == (8192, 4) and w["w_qkv"].shape == (8192, 2048)
    assert w["w_out"].shape == (2048, 4096) and w["A_log"].dtype == np.float32
    assert 0.0 <= w["A_log"].min() and w["A_log"].max() < np.log(16.0)
    std = synth.bf16_to_f32(w["w_z"]).std()
    assert abs(std - 0.02) < 1e-3
