"""Generate the golden fixtures under tests/golden/ (run from the repo root).

    python tests/golden/make_golden.py

Recurrence cases ("ref_*") come from the reference's own Metal kernel body
(src/models/metal_gdn.rs:10-67) compiled for the CPU by oracle/build.py; they
pin the oracle's recurrence restatement.  Layer cases ("orc_*") come from the
oracle restatement of the MLX layer (there is no runnable MLX here); they pin
the oracle against later edits.  Inputs are regenerated from the seeded
generator (qwen-mlx_b200/synth.py), so only outputs are stored: the SHA-256 of
every output array plus a strided sample of its values (golden.npz).
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import __graft_entry__ as ge  # noqa: E402

OUT_DIR = Path(__file__).resolve().parent
SAMPLE_STRIDE = 127


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def recurrence_inputs(case: dict):
    S = ge.load_package().synth
    B, T, hk, hv, dk, dv = (case[k] for k in ("B", "T", "hk", "hv", "dk", "dv"))
    tag = case["name"]
    seed = case["seed"]
    q = S.normal(seed, tag + "q", B * T * hk * dk).reshape(B, T, hk, dk)
    k = S.normal(seed, tag + "k", B * T * hk * dk).reshape(B, T, hk, dk)
    # q, k as the layer feeds them: RMS-normalised with gains 1/dk and dk^-1/2
    q = q / np.sqrt((q * q).mean(-1, keepdims=True) + 1e-6) / dk
    k = k / np.sqrt((k * k).mean(-1, keepdims=True) + 1e-6) / np.sqrt(dk)
    q = S.f32_to_bf16(q.astype(np.float32))
    k = S.f32_to_bf16(k.astype(np.float32))
    v = S.normal_bf16(seed, tag + "v", (B, T, hv, dv))
    g = S.uniform(seed, tag + "g", B * T * hv, 0.5, 1.0).astype(np.float32).reshape(B, T, hv)
    beta = S.f32_to_bf16(S.uniform(seed, tag + "beta", B * T * hv).astype(np.float32)).reshape(B, T, hv)
    if case["zero_state"]:
        st = np.zeros((B, hv, dv, dk), np.float32)
    else:
        st = (S.normal(seed, tag + "state", B * hv * dv * dk) * 0.1).astype(np.float32).reshape(B, hv, dv, dk)
    return q, k, v, g, beta, st


RECURRENCE_CASES = [
    # config-1 shape: one sequence, 64 tokens, zero state
    dict(name="ref_cfg1_T64", B=1, T=64, hk=16, hv=32, dk=128, dv=128, seed=0, zero_state=True),
    dict(name="ref_b3_t4_gqa2", B=3, T=4, hk=2, hv=4, dk=128, dv=128, seed=0, zero_state=False),
    dict(name="ref_b2_t9_gqa2", B=2, T=9, hk=1, hv=2, dk=128, dv=128, seed=0, zero_state=False),
    dict(name="ref_b4_t1_decode", B=4, T=1, hk=16, hv=32, dk=128, dv=128, seed=0, zero_state=False),
]


def layer_case_inputs(case: dict):
    S = ge.load_package().synth
    cfg = S.GdnConfig(n_layers=1)
    lens = case["lens"]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    inp = S.step_inputs(cfg, int(cu[-1]), seed=case["seed"], tag=case["name"])
    if case["zero_state"]:
        conv = np.zeros((len(lens), cfg.conv_k - 1, cfg.conv_dim), np.uint16)
        rec = np.zeros((len(lens), cfg.hv, cfg.dv, cfg.dk), np.float32)
    else:
        conv, rec = S.random_states(cfg, len(lens), seed=case["seed"], tag=case["name"])
    w = S.layer_weights(cfg, case.get("layer", 0), with_proj=False)
    return cfg, w, inp, conv, rec, cu


LAYER_CASES = [
    dict(name="orc_decode_b8", lens=[1] * 8, seed=0, zero_state=False),
    dict(name="orc_ragged", lens=[1, 3, 1, 5, 0, 2, 17], seed=0, zero_state=False),
    dict(name="orc_prefill_zero", lens=[33], seed=0, zero_state=True),
]


def mixer_case(n_steps=64):
    """Config 1: one layer with projections, B=1, zero state, n_steps decode steps of x ~ N(0,1)."""
    S = ge.load_package().synth
    cfg = S.GdnConfig(n_layers=1)
    w = S.layer_weights(cfg, 0, with_proj=True)
    x = S.normal_bf16(0, "cfg1_x", (n_steps, cfg.hidden))
    return cfg, w, x


def run_all(O):
    outputs = {}
    for case in RECURRENCE_CASES:
        q, k, v, g, beta, st = recurrence_inputs(case)
        args = (case["T"], case["B"], case["hk"], case["hv"], case["dk"], case["dv"])
        res = O.ref_recurrence(q, k, v, g, beta, st, *args)
        if res is None:
            raise RuntimeError("oracle/_ref/libgdn_metal_ref.so is missing: run oracle/build.py with the reference tree")
        outputs[case["name"]] = {"y": res[0], "state": res[1]}
    for case in LAYER_CASES:
        cfg, w, inp, conv, rec, cu = layer_case_inputs(case)
        out, cs, rs, y = O.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv, rec, cu, want_y=True)
        outputs[case["name"]] = {"out": out, "y": y, "conv": cs, "rec": rs}
    cfg, w, x = mixer_case()
    conv = np.zeros((1, cfg.conv_k - 1, cfg.conv_dim), np.uint16)
    rec = np.zeros((1, cfg.hv, cfg.dv, cfg.dk), np.float32)
    outs = []
    for t in range(x.shape[0]):
        o, conv, rec = O.mixer_step(cfg, w, x[t:t + 1], conv, rec, np.array([0, 1], np.int32))
        outs.append(o)
    outputs["orc_cfg1_mixer_64steps"] = {"out": np.concatenate(outs), "conv": conv, "rec": rec}
    return outputs


def main():
    O = ge.load_oracle()
    outputs = run_all(O)
    manifest = {"sample_stride": SAMPLE_STRIDE, "cases": {}}
    samples = {}
    for name, arrs in outputs.items():
        manifest["cases"][name] = {k: {"sha256": sha(a), "shape": list(a.shape), "dtype": str(a.dtype)}
                                   for k, a in arrs.items()}
        for k, a in arrs.items():
            samples[f"{name}/{k}"] = np.ascontiguousarray(a).reshape(-1)[::SAMPLE_STRIDE]
    manifest["recurrence_cases"] = RECURRENCE_CASES
    manifest["layer_cases"] = LAYER_CASES
    (OUT_DIR / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    np.savez_compressed(OUT_DIR / "golden.npz", **samples)
    print(f"wrote {len(outputs)} cases")


if __name__ == "__main__":
    main()
