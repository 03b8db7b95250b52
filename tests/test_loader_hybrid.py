"""The checkpoint loader for the attention and MoE layers (row f4): a small Qwen3.5-layout checkpoint with
attention every 4th layer and a MoE block in every layer, written here 4-bit quantized (router and
shared-expert gate included, as the reference's whole-model quantize does) and in bf16."""
from __future__ import annotations

import importlib
import json

import numpy as np
import pytest

H, NH, NKV, HD, E, K, I, IS, LAYERS, INTERVAL = 256, 4, 2, 64, 4, 2, 128, 64, 4, 4


@pytest.fixture
def loader(pkg):
    return importlib.import_module("qwen_mlx_b200.loader")


def _write(synth, loader, d, quantized: bool):
    cfg = {"text_config": {"hidden_size": H, "num_hidden_layers": LAYERS, "full_attention_interval": INTERVAL,
                           "num_attention_heads": NH, "num_key_value_heads": NKV, "head_dim": HD,
                           "partial_rotary_factor": 0.25, "rope_theta": 1e6, "num_experts": E,
                           "num_experts_per_tok": K, "moe_intermediate_size": I, "shared_expert_intermediate_size": IS},
           "rms_norm_eps": 1e-6}
    if quantized:
        cfg["quantization"] = {"group_size": 64, "bits": 4}
    t, bf16, ref = {}, set(), {}

    def put(name, w):   # w: bf16 [rows, cols] (or [E, rows, cols])
        if quantized:
            flat = w.reshape(-1, w.shape[-1])
            q, s, b = synth.quantize_q4(flat)
            lead = w.shape[:-1]
            t[name + ".weight"] = q.reshape(*lead, -1)
            t[name + ".scales"], t[name + ".biases"] = s.reshape(*lead, -1), b.reshape(*lead, -1)
            bf16.update({name + ".scales", name + ".biases"})
            ref[name] = (q, s, b)
        else:
            t[name + ".weight"] = w
            bf16.add(name + ".weight")
            ref[name] = w

    for l in range(LAYERS):
        pl = f"language_model.model.layers.{l}"
        if (l + 1) % INTERVAL == 0:
            for n, shape in (("q_proj", (2 * NH * HD, H)), ("k_proj", (NKV * HD, H)), ("v_proj", (NKV * HD, H)),
                             ("o_proj", (H, NH * HD))):
                put(f"{pl}.self_attn.{n}", synth.normal_bf16(l, n, shape, 0.02))
            for n in ("q_norm", "k_norm"):
                t[f"{pl}.self_attn.{n}.weight"] = synth.normal_bf16(l, n, (HD,))
                bf16.add(f"{pl}.self_attn.{n}.weight")
            t[f"{pl}.input_layernorm.weight"] = synth.normal_bf16(l, "pre", (H,))
            bf16.add(f"{pl}.input_layernorm.weight")
        t[f"{pl}.post_attention_layernorm.weight"] = synth.normal_bf16(l, "post", (H,))
        bf16.add(f"{pl}.post_attention_layernorm.weight")
        put(f"{pl}.mlp.gate", synth.normal_bf16(l, "router", (E, H), 0.02))
        put(f"{pl}.mlp.shared_expert_gate", synth.normal_bf16(l, "sg", (1, H), 0.02))
        put(f"{pl}.mlp.switch_mlp.gate_proj", synth.normal_bf16(l, "eg", (E, I, H), 0.02))
        put(f"{pl}.mlp.switch_mlp.up_proj", synth.normal_bf16(l, "eu", (E, I, H), 0.02))
        put(f"{pl}.mlp.switch_mlp.down_proj", synth.normal_bf16(l, "ed", (E, H, I), 0.02))
        put(f"{pl}.mlp.shared_expert.gate_proj", synth.normal_bf16(l, "sgp", (IS, H), 0.02))
        put(f"{pl}.mlp.shared_expert.up_proj", synth.normal_bf16(l, "sup", (IS, H), 0.02))
        put(f"{pl}.mlp.shared_expert.down_proj", synth.normal_bf16(l, "sdp", (H, IS), 0.02))
    loader.save_safetensors(d / "model.safetensors", t, bf16=bf16)
    (d / "config.json").write_text(json.dumps(cfg))
    return t, ref


def test_attention_layers_load(synth, loader, tmp_path):
    t, ref = _write(synth, loader, tmp_path, quantized=True)
    a, layers, ws = loader.load_attention_layers(tmp_path, max_ctx=512)
    assert layers == [3]
    assert a == dict(n_heads=NH, n_kv_heads=NKV, head_dim=HD, rotary_dim=16, rope_theta=1e6, rms_norm_eps=1e-6,
                     max_ctx=512)
    w = ws[0]
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        for got, want in zip(w[n], ref[f"language_model.model.layers.3.self_attn.{n}"]):
            assert np.array_equal(got, want)
    assert np.array_equal(w["q_norm_w"], t["language_model.model.layers.3.self_attn.q_norm.weight"])
    assert np.array_equal(w["post_w"], t["language_model.model.layers.3.post_attention_layernorm.weight"])


def test_moe_layers_load_quantized(synth, loader, oracle, tmp_path):
    t, ref = _write(synth, loader, tmp_path, quantized=True)
    m, ws = loader.load_moe_layers(tmp_path)
    assert m == dict(hidden=H, n_experts=E, top_k=K, moe_inter=I, shared_inter=IS, norm_topk_prob=True)
    assert len(ws) == LAYERS
    w, p = ws[2], "language_model.model.layers.2.mlp"
    # experts stacked by rows, bit for bit
    q, s, b = ref[f"{p}.switch_mlp.down_proj"]
    assert w["down"]["q"].shape == (E * H, I // 8) and np.array_equal(w["down"]["q"], q)
    assert np.array_equal(w["down"]["scales"], s) and np.array_equal(w["down"]["biases"], b)
    assert np.array_equal(w["sh_up"]["q"], ref[f"{p}.shared_expert.up_proj"][0])
    # the router and the shared-expert gate dequantized to bf16 by the projections' rule
    q, s, b = ref[f"{p}.gate"]
    assert np.array_equal(w["router"], oracle.q4_dequantize(q, s, b))
    q, s, b = ref[f"{p}.shared_expert_gate"]
    assert np.array_equal(w["shared_gate"], oracle.q4_dequantize(q, s, b)[0])


def test_moe_layers_bf16_checkpoint_rejected(synth, loader, tmp_path):
    _write(synth, loader, tmp_path, quantized=False)
    with pytest.raises(ValueError, match="4-bit"):
        loader.load_moe_layers(tmp_path)
    a, layers, ws = loader.load_attention_layers(tmp_path)   # bf16 attention projections load as they are
    assert ws[0]["q_proj"].shape == (2 * NH * HD, H)


def test_dequantize_8bit(synth, loader):
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 256, size=(3, 128), dtype=np.uint32)
    words = (codes.reshape(3, 32, 4) << (np.arange(4, dtype=np.uint32) * 8)).sum(axis=2, dtype=np.uint64)
    s = synth.f32_to_bf16(np.full((3, 2), 0.5, np.float32))
    b = synth.f32_to_bf16(np.full((3, 2), -3.0, np.float32))
    got = synth.bf16_to_f32(loader.dequantize(words.astype(np.uint32), s, b, 8, 64))
    assert np.array_equal(got, codes.astype(np.float32) * 0.5 - 3.0)
