"""A checkpoint in the reference's layout, loaded by gdn.load_mixer_weights (4-bit MLX projections), drives
the residual GDN stack on the GPU; the oracle runs the same stack on the dequantized weights.  Tolerance as in
test_gpu_mixer.py: max(1e-3, 2 x the oracle's own spread over valid GEMM accumulation orders)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ALT_ORDERS, order_noise, rel_l2, with_order
from test_loader import _write_checkpoint

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = 1e-3


@pytest.mark.parametrize("first", [[7, 40, 2], [7, 90, 2]])
def test_quantized_checkpoint_stack_matches_oracle(gdn, synth, oracle, tmp_path, first):
    """First step 49 tokens (4-bit weight-streaming kernel) or 99 tokens (more than 64: the weight is expanded
    to bf16 once per projection and multiplied by the library GEMM), then two decode steps."""
    import importlib
    loader = importlib.import_module("qwen_mlx_b200.loader")
    _write_checkpoint(synth, loader, tmp_path, quantized=True, seed=7)
    cfg, layers, mws = gdn.load_mixer_weights(tmp_path, DEV)
    _, _, raw = loader.load_gdn_layers(tmp_path)
    ws = []
    for w in raw:   # the oracle's weights: each projection dequantized (MLX rounding), split back into parts
        d_in = oracle.q4_dequantize(*w["q4_in"])
        D, Z, hv = cfg.conv_dim, cfg.z_dim, cfg.hv
        o = dict(w)
        o["w_qkv"], o["w_z"], o["w_b"], o["w_a"] = d_in[:D], d_in[D:D + Z], d_in[D + Z:D + Z + hv], d_in[D + Z + hv:]
        o["w_out"] = oracle.q4_dequantize(*w["q4_out"])
        ws.append(o)
    slots = np.array([3, 0, 5], np.int32)
    L, n = cfg.n_layers, len(slots)
    cs = np.zeros((L, n, cfg.conv_k - 1, cfg.conv_dim), np.uint16)
    rs = np.zeros((L, n, cfg.hv, cfg.dv, cfg.dk), np.float32)
    alt = {o: (cs.copy(), rs.copy()) for o in ALT_ORDERS}
    f = synth.bf16_to_f32
    with gdn.StatePool(cfg, n_slots=8, device=0) as pool:
        for it, lens in enumerate([first, [1, 1, 1], [1, 1, 1]]):
            cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
            N = int(cu[-1])
            h0 = synth.normal_bf16(50 + it, "ck_h", (N, cfg.hidden))
            hd = gdn.bf16_to_device(h0, DEV)
            pool.stack_step(mws, hd, torch.from_numpy(slots).to(DEV), torch.from_numpy(cu).to(DEV), N)
            torch.cuda.synchronize()
            h_alts = []
            for o in ALT_ORDERS:
                ca, ra = alt[o]
                h_o, ca, ra = with_order(oracle, o, lambda: oracle.stack_step(cfg, ws, h0, ca, ra, cu))
                alt[o] = (ca, ra)
                h_alts.append(h_o)
            h_ref, cs, rs = oracle.stack_step(cfg, ws, h0, cs, rs, cu)
            tol = max(TOL, 2 * order_noise(h_ref, h_alts, f))
            assert rel_l2(f(gdn.bf16_to_host(hd)), f(h_ref)) < tol, f"step {it}"
        assert pool.check() == 0
