"""The oracle against the committed golden fixtures (tests/golden/, made by make_golden.py).

Recurrence cases were produced by the reference's own Metal kernel body
(metal_gdn.rs:10-67) compiled for the CPU; matching their SHA-256 pins the
oracle's recurrence to the reference bit for bit.  Layer cases pin the oracle's
restatement of the MLX layer against later edits.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden as mg  # noqa: E402

MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())
SAMPLES = np.load(GOLDEN / "golden.npz")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _check(name, arrays):
    exp = MANIFEST["cases"][name]
    stride = MANIFEST["sample_stride"]
    for k, a in arrays.items():
        assert list(a.shape) == exp[k]["shape"], (name, k)
        assert np.array_equal(a.reshape(-1)[::stride], SAMPLES[f"{name}/{k}"]), (name, k, "sample")
        assert _sha(a) == exp[k]["sha256"], (name, k, "sha256")


def test_manifest_covers_all_cases():
    names = {c["name"] for c in mg.RECURRENCE_CASES} | {c["name"] for c in mg.LAYER_CASES}
    names.add("orc_cfg1_mixer_64steps")
    assert names == set(MANIFEST["cases"])


@pytest.mark.parametrize("case", mg.RECURRENCE_CASES, ids=lambda c: c["name"])
def test_oracle_recurrence_matches_reference_golden(oracle, case):
    q, k, v, g, beta, st = mg.recurrence_inputs(case)
    y, s = oracle.recurrence(q, k, v, g, beta, st, case["T"], case["B"], case["hk"], case["hv"], case["dk"],
                             case["dv"])
    _check(case["name"], {"y": y, "state": s})


@pytest.mark.parametrize("case", mg.LAYER_CASES, ids=lambda c: c["name"])
def test_oracle_layer_matches_golden(oracle, case):
    cfg, w, inp, conv, rec, cu = mg.layer_case_inputs(case)
    out, cs, rs, y = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv, rec, cu, want_y=True)
    _check(case["name"], {"out": out, "y": y, "conv": cs, "rec": rs})


def test_oracle_config1_mixer_matches_golden(oracle):
    cfg, w, x = mg.mixer_case()
    conv = np.zeros((1, cfg.conv_k - 1, cfg.conv_dim), np.uint16)
    rec = np.zeros((1, cfg.hv, cfg.dv, cfg.dk), np.float32)
    outs = []
    for t in range(x.shape[0]):
        o, conv, rec = oracle.mixer_step(cfg, w, x[t:t + 1], conv, rec, np.array([0, 1], np.int32))
        outs.append(o)
    _check("orc_cfg1_mixer_64steps", {"out": np.concatenate(outs), "conv": conv, "rec": rec})


def test_oracle_long_prompt_layer_matches_full_size_golden(oracle):
    """The oracle on the long-prompt prefill set (30,016 tokens, one full-width layer) reproduces the
    committed full-size fixture bit for bit (tests/golden/make_golden_full.py)."""
    import make_golden_full as mgf
    meta = json.loads((GOLDEN / "manifest_full.json").read_text())["cfg4_layer"]
    cfg, w, inp, cu = mgf.cfg4_inputs()
    out, cs, rs = mgf.run_cfg4(oracle, cfg, w, inp, cu)
    assert _sha(out) == meta["sha256"]["out"]
    assert _sha(rs) == meta["sha256"]["rec"]
    assert _sha(cs) == meta["sha256"]["conv"]
    full = np.load(GOLDEN / "golden_full.npz")
    for k, a in mgf.cfg4_samples(out, rs, cu).items():
        assert np.array_equal(a, full[f"cfg4_layer/{k}"]), k
