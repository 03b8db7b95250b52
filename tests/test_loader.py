"""The checkpoint loader (f3 row): a small Qwen3.5-layout checkpoint written here (nested text_config,
two safetensors shards behind an index, bf16 and MLX 4-bit variants) loads into the package's weight dicts
with the reference's layer selection, merge order and conv re-layout."""
from __future__ import annotations

import json

import numpy as np
import pytest

HIDDEN, HK, HV, DK, LAYERS, INTERVAL = 256, 2, 4, 128, 8, 4


def _write_checkpoint(synth, loader, d, quantized: bool, seed: int = 1):
    cfg = {"model_type": "qwen3_5_moe",
           "text_config": {"hidden_size": HIDDEN, "num_hidden_layers": LAYERS, "full_attention_interval": INTERVAL,
                           "linear_num_key_heads": HK, "linear_num_value_heads": HV, "linear_key_head_dim": DK,
                           "linear_value_head_dim": DK, "linear_conv_kernel_dim": 4},
           "rms_norm_eps": 1e-6}
    if quantized:
        cfg["quantization"] = {"group_size": 64, "bits": 4}
    D, Z = 2 * HK * DK + HV * DK, HV * DK
    shards = [{}, {}]
    bf16 = set()
    ref = {}
    for l in range(LAYERS):
        if (l + 1) % INTERVAL == 0:
            continue
        p = f"language_model.model.layers.{l}.linear_attn"
        sh = shards[l % 2]
        projs = {"in_proj_qkv": (D, HIDDEN), "in_proj_z": (Z, HIDDEN), "in_proj_a": (HV, HIDDEN),
                 "in_proj_b": (HV, HIDDEN), "out_proj": (HIDDEN, Z)}
        for name, shape in projs.items():
            w = synth.normal_bf16(seed + l, f"{name}", shape, 0.02)
            if quantized:
                wq, sc, bi = synth.quantize_q4(w)
                sh[f"{p}.{name}.weight"], sh[f"{p}.{name}.scales"], sh[f"{p}.{name}.biases"] = wq, sc, bi
                bf16 |= {f"{p}.{name}.scales", f"{p}.{name}.biases"}
                ref[(l, name)] = (wq, sc, bi)
            else:
                sh[f"{p}.{name}.weight"] = w
                bf16.add(f"{p}.{name}.weight")
                ref[(l, name)] = w
        conv = synth.normal_bf16(seed + l, "conv", (D, 4, 1), 0.02)
        sh[f"{p}.conv1d.weight"] = conv
        sh[f"{p}.A_log"] = np.linspace(0.1, 2.0, HV).astype(np.float32)
        sh[f"{p}.dt_bias"] = synth.f32_to_bf16(np.linspace(-1, 1, HV).astype(np.float32))   # stored bf16
        sh[f"{p}.norm.weight"] = synth.f32_to_bf16(np.full(DK, 1.5, np.float32))
        sh[f"language_model.model.layers.{l}.input_layernorm.weight"] = synth.f32_to_bf16(np.ones(HIDDEN, np.float32))
        bf16 |= {f"{p}.conv1d.weight", f"{p}.dt_bias", f"{p}.norm.weight",
                 f"language_model.model.layers.{l}.input_layernorm.weight"}
        ref[(l, "conv")] = conv
    names = ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]
    wmap = {}
    for sh, fn in zip(shards, names):
        loader.save_safetensors(d / fn, sh, bf16=bf16 & set(sh))
        wmap.update({k: fn for k in sh})
    (d / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wmap}))
    (d / "config.json").write_text(json.dumps(cfg))
    return ref


@pytest.fixture
def loader(pkg):
    import importlib
    return importlib.import_module("qwen_mlx_b200.loader")


def test_safetensors_round_trip(synth, loader, tmp_path):
    t = {"a": np.arange(12, dtype=np.float32).reshape(3, 4), "b": np.array([1, 2, 3], np.uint32),
         "c": synth.f32_to_bf16(np.array([1.5, -2.0], np.float32))}
    loader.save_safetensors(tmp_path / "x.safetensors", t, bf16={"c"})
    st = loader.SafeTensors(tmp_path / "x.safetensors")
    assert st.dtype("c") == "BF16" and st.dtype("a") == "F32"
    for k, v in t.items():
        assert np.array_equal(st.get(k), v)


@pytest.mark.parametrize("quantized", [False, True])
def test_loader_selection_merge_and_layout(synth, loader, tmp_path, quantized):
    ref = _write_checkpoint(synth, loader, tmp_path, quantized)
    cfg, layers, ws = loader.load_gdn_layers(tmp_path)
    assert layers == [0, 1, 2, 4, 5, 6]                 # (l + 1) % 4 != 0
    assert (cfg.hidden, cfg.hk, cfg.hv, cfg.n_layers, cfg.eps) == (HIDDEN, HK, HV, 6, 1e-6)
    for l, w in zip(layers, ws):
        assert np.array_equal(w["conv_w"], ref[(l, "conv")].reshape(-1, 4))
        assert w["dt_bias"].dtype == np.float32 and np.allclose(w["dt_bias"], np.linspace(-1, 1, HV), atol=1e-2)
        assert w["dt_bias_bf16"] is True                 # stored bf16: the bf16 gate arithmetic applies
        assert np.all(synth.bf16_to_f32(w["norm_w"]) == 1.5)
        order = ["in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a"]   # [qkv; z] then [b; a]
        if quantized:
            for i in range(3):
                assert np.array_equal(w["q4_in"][i], np.concatenate([ref[(l, n)][i] for n in order]))
                assert np.array_equal(w["q4_out"][i], ref[(l, "out_proj")][i])
        else:
            assert np.array_equal(w["w_qkv"], ref[(l, "in_proj_qkv")])
            assert np.array_equal(w["w_b"], ref[(l, "in_proj_b")]) and np.array_equal(w["w_a"], ref[(l, "in_proj_a")])
            assert np.array_equal(w["w_out"], ref[(l, "out_proj")])


def test_loader_rejects_wrong_shapes(synth, loader, tmp_path):
    _write_checkpoint(synth, loader, tmp_path, False)
    cfg = json.loads((tmp_path / "config.json").read_text())
    cfg["text_config"]["linear_num_value_heads"] = 8                      # disagrees with the tensors
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError):
        loader.load_gdn_layers(tmp_path)
