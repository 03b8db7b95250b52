"""Host-side mirror of the reference GDN interfaces over the C ABI.

  gated_delta_kernel(...)      -- metal_gdn.rs:170-218, same argument meaning,
                                  functional (returns y and a new state)
  StatePool                    -- the slot-indexed device state pool that replaces
                                  Qwen35State + stack/unstack (mlx_executor.rs:19-130)
  StatePool.layer_step(...)    -- the fused layer body of GatedDeltaNet::forward_with_cache
                                  between the projections (qwen3_5.rs:588-665)
  beta_g(...)                  -- compiled_beta_g (compiled_ops.rs:68-94)

torch is used only to hold device memory and streams; every computation runs
in libgdn_b200.so.  bf16 tensors are torch.bfloat16 on the device and uint16
bit patterns on the host.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import abi
from .synth import GdnConfig


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream):
    if stream is None:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, torch.cuda.Stream):
        return C.c_void_p(stream.cuda_stream)
    return C.c_void_p(int(stream))


def bf16_to_device(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def bf16_to_host(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def f32_to_device(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def _check_dev(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def gated_delta_kernel(q, k, v, g, beta, state, seq_len, batch, hk, hv, dk, dv, out_state=None, stream=None):
    """Gated delta recurrence with the argument meaning of metal_gdn.rs:170-173.

    q, k [B,T,Hk,dk] bf16; v [B,T,Hv,dv] bf16; g [B,T,Hv] f32; beta [B,T,Hv] bf16;
    state [B,Hv,dv,dk] f32.  Returns (y [B,T,Hv,dv] bf16, new_state [B,Hv,dv,dk] f32);
    `state` is left untouched unless `out_state is state` (in-place update).
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta), ("state", state)):
        _check_dev(t, name)
    y = torch.empty((batch, seq_len, hv, dv), dtype=torch.bfloat16, device=q.device)
    new_state = torch.empty_like(state) if out_state is None else out_state
    abi.call("gdn_gated_delta_kernel", _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), seq_len, batch,
             hk, hv, dk, dv, _ptr(y), _ptr(new_state), _stream(stream))
    return y, new_state


def beta_g(ab, A_log, dt_bias, hv, stream=None, dt_bias_bf16=False):
    """compiled_beta_g over an [N, >=2*Hv] (b | a) buffer: returns (beta bf16 [N,Hv], g f32 [N,Hv]).
    dt_bias_bf16: dt_bias is a bf16 parameter (given widened to f32); a + dt_bias and its exp round to bf16."""
    n = ab.shape[0]
    beta = torch.empty((n, hv), dtype=torch.bfloat16, device=ab.device)
    g = torch.empty((n, hv), dtype=torch.float32, device=ab.device)
    abi.call("gdn_beta_g_ex", _ptr(ab), ab.stride(0), n, hv, _ptr(A_log), _ptr(dt_bias), 1 if dt_bias_bf16 else 0,
             _ptr(beta), _ptr(g), _stream(stream))
    return beta, g


class LayerWeights:
    """Device copies of one layer's step parameters (conv_w [D,K], A_log, dt_bias, norm_w)."""

    def __init__(self, w: dict, device):
        self.conv_w = bf16_to_device(w["conv_w"], device)
        self.A_log = f32_to_device(w["A_log"], device)
        self.dt_bias = f32_to_device(w["dt_bias"], device)
        self.norm_w = bf16_to_device(w["norm_w"], device)
        # a checkpoint that stores dt_bias in bf16 (loader: "dt_bias_bf16") gets the bf16 gate arithmetic
        self.dt_bias_bf16 = bool(w.get("dt_bias_bf16", False))
        self.c = abi.GdnLayerWeightsC(self.conv_w.data_ptr(), self.A_log.data_ptr(), self.dt_bias.data_ptr(),
                                      self.norm_w.data_ptr(), 1 if self.dt_bias_bf16 else 0)


def tile_weight(w, stream=None):
    """The tiled copy (gdn_weight_tile) of a row-major bf16 device weight w [n_out, n_in]: the layout
    the weight-streaming projection kernel reads.  Returns a uint8 device tensor."""
    n_out, n_in = w.shape
    t = torch.empty(int(abi.lib().gdn_weight_tile_bytes(n_out, n_in)), dtype=torch.uint8, device=w.device)
    abi.call("gdn_weight_tile", n_out, n_in, _ptr(w), _ptr(t), _stream(stream))
    return t


def tile_weight_q4(w_q, scales, biases, stream=None):
    """The tiled copy (gdn_weight_tile_q4) of an MLX 4-bit weight given as device tensors w_q [n_out,
    n_in/8] (int32 holding the uint32 words), scales and biases [n_out, n_in/64] bf16."""
    n_out, n_in = w_q.shape[0], w_q.shape[1] * 8
    t = torch.empty(int(abi.lib().gdn_weight_tile_q4_bytes(n_out, n_in)), dtype=torch.uint8, device=w_q.device)
    abi.call("gdn_weight_tile_q4", n_out, n_in, _ptr(w_q), _ptr(scales), _ptr(biases), _ptr(t), _stream(stream))
    return t


def q4_to_device(w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray, device):
    """Upload an MLX 4-bit weight (numpy uint32 words, bf16 bit patterns) and tile it."""
    wq = torch.from_numpy(np.ascontiguousarray(w_q, np.uint32).view(np.int32)).to(device)
    return tile_weight_q4(wq, bf16_to_device(scales, device), bf16_to_device(biases, device))


class MixerWeights:
    """Device copies of one whole mixer layer: step parameters, merged in-projection
    [qkv | z | b | a] rows (the reference's merged order), out-projection and the
    decoder input-norm gain.

    tiled=True adds the bf16 tiled copies (calls of at most 64 tokens run the projections on the
    weight-streaming tensor-core kernel).  q4=(w_in_q, w_out_q), each a (w_q, scales, biases) MLX
    4-bit weight (synth.quantize_q4 or a quantized checkpoint), makes the projections 4-bit for every
    call; the row-major bf16 weights are then not uploaded."""

    def __init__(self, w: dict, device, tiled: bool = False, q4=None):
        self.step = LayerWeights(w, device)
        self.pre_w = bf16_to_device(w["pre_w"], device)
        self.w_in = self.w_out = self.w_in_tiles = self.w_out_tiles = self.w_in_q4 = self.w_out_q4 = None
        if q4 is not None:
            self.w_in_q4 = q4_to_device(*q4[0], device)
            self.w_out_q4 = q4_to_device(*q4[1], device)
        else:
            w_in = np.concatenate([w["w_qkv"], w["w_z"], w["w_b"], w["w_a"]], axis=0)
            self.w_in = bf16_to_device(w_in, device)
            self.w_out = bf16_to_device(w["w_out"], device)
            if tiled:
                self.w_in_tiles = tile_weight(self.w_in)
                self.w_out_tiles = tile_weight(self.w_out)

        def p(t):
            return t.data_ptr() if t is not None else None

        self.c = abi.GdnMixerWeightsC(self.step.c, p(self.w_in), p(self.w_out), self.pre_w.data_ptr(),
                                      p(self.w_in_tiles), p(self.w_out_tiles), p(self.w_in_q4), p(self.w_out_q4))


def load_mixer_weights(model_dir, device, tiled: bool = False):
    """(GDN shapes, linear-layer indices, [MixerWeights]) of a checkpoint directory in the reference's layout
    (loader.load_gdn_layers): 4-bit projections for a quantized checkpoint, bf16 otherwise."""
    from . import loader
    cfg, layers, ws = loader.load_gdn_layers(model_dir)
    mws = [MixerWeights(w, device, tiled=tiled, q4=(w["q4_in"], w["q4_out"]) if "q4_in" in w else None) for w in ws]
    return cfg, layers, mws


def merged_in_proj(w: dict) -> np.ndarray:
    """The merged in-projection rows [qkv | z | b | a] of a synthetic weight dict."""
    return np.concatenate([w["w_qkv"], w["w_z"], w["w_b"], w["w_a"]], axis=0)


class StatePool:
    """Slot-indexed device pool of GDN states for `cfg.n_layers` layers."""

    def __init__(self, cfg: GdnConfig, n_slots: int, device: int = 0):
        self.cfg = cfg
        self.n_slots = n_slots
        self.device = device
        c = abi.GdnConfigC(cfg.hidden, cfg.hk, cfg.hv, cfg.dk, cfg.dv, cfg.conv_k, cfg.n_layers, cfg.eps)
        h = C.c_void_p()
        abi.call("gdn_pool_create", device, C.byref(c), n_slots, C.byref(h))
        self.h = h

    def close(self):
        if self.h is not None and self.h.value:
            abi.call("gdn_pool_destroy", self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---------------------------------------------------------------- state
    def nbytes(self) -> int:
        n = C.c_size_t()
        abi.call("gdn_pool_bytes", self.h, C.byref(n))
        return int(n.value)

    def reserve_tokens(self, max_tokens: int):
        abi.call("gdn_pool_reserve_tokens", self.h, int(max_tokens))

    def layer_state_ptrs(self, layer: int):
        rec, conv = C.c_void_p(), C.c_void_p()
        abi.call("gdn_pool_layer_state", self.h, layer, C.byref(rec), C.byref(conv))
        return rec.value, conv.value

    def reset(self, slots, stream=None):
        arr = np.ascontiguousarray(slots, dtype=np.int32)
        abi.call("gdn_slot_reset", self.h, arr.ctypes.data_as(C.c_void_p), len(arr), _stream(stream))

    def export(self, slot: int, layer: int):
        cfg = self.cfg
        rec = np.zeros((cfg.hv, cfg.dv, cfg.dk), np.float32)
        conv = np.zeros((cfg.conv_k - 1, cfg.conv_dim), np.uint16)
        torch.cuda.synchronize(self.device)
        abi.call("gdn_slot_export", self.h, slot, layer, rec.ctypes.data_as(C.c_void_p),
                 conv.ctypes.data_as(C.c_void_p))
        return rec, conv

    def import_(self, slot: int, layer: int, rec=None, conv=None):
        torch.cuda.synchronize(self.device)
        r = np.ascontiguousarray(rec, dtype=np.float32) if rec is not None else None
        c = np.ascontiguousarray(conv, dtype=np.uint16) if conv is not None else None
        abi.call("gdn_slot_import", self.h, slot, layer, r.ctypes.data_as(C.c_void_p) if r is not None else None,
                 c.ctypes.data_as(C.c_void_p) if c is not None else None)

    def check(self, reset: bool = True) -> int:
        f = C.c_int32()
        abi.call("gdn_pool_check", self.h, C.byref(f), 1 if reset else 0)
        return int(f.value)

    def validate(self, slot_ids, cu_seqlens, n_tokens=None):
        s = np.ascontiguousarray(slot_ids, dtype=np.int32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        n_tokens = int(cu[-1]) if n_tokens is None else n_tokens
        abi.call("gdn_validate_batch", self.h, s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                 len(s), n_tokens)

    # ---------------------------------------------------------------- compute
    def layer_step(self, layer: int, w: LayerWeights, qkv, z, ab, out, slot_ids, cu_seqlens, n_tokens: int,
                   stream=None, flags: int = 0):
        """Fused layer step; qkv/z/ab/out are [N, ld] device tensors, tables are device int32.  flags:
        abi.GDN_STEP_TABLES_STABLE for the later layers of a step (gdn_layer_step_ex)."""
        io = abi.GdnStepIOC(qkv.data_ptr(), qkv.stride(0), z.data_ptr(), z.stride(0), ab.data_ptr(), ab.stride(0),
                            out.data_ptr(), out.stride(0))
        if flags:
            abi.call("gdn_layer_step_ex", self.h, layer, C.byref(w.c), C.byref(io), _ptr(slot_ids), _ptr(cu_seqlens),
                     slot_ids.numel(), n_tokens, flags, _stream(stream))
        else:
            abi.call("gdn_layer_step", self.h, layer, C.byref(w.c), C.byref(io), _ptr(slot_ids), _ptr(cu_seqlens),
                     slot_ids.numel(), n_tokens, _stream(stream))

    def layer_step_raw(self, layer: int, w_c, io_c, slot_ptr, cu_ptr, n_seq, n_tokens, stream_ptr):
        """Same as layer_step with prebuilt ctypes arguments (no per-call Python allocation)."""
        rc = abi.lib().gdn_layer_step(self.h, layer, w_c, io_c, slot_ptr, cu_ptr, n_seq, n_tokens, stream_ptr)
        if rc:
            abi.check(rc, "gdn_layer_step")

    def linear(self, x, w, y, stream=None):
        """y = x @ w.T (bf16, f32 accumulation): x [M, K], w [N, K], y [M, N] device tensors."""
        abi.call("gdn_linear", self.h, x.shape[0], w.shape[0], w.shape[1], _ptr(x), x.stride(0), _ptr(w), _ptr(y),
                 y.stride(0), _stream(stream))

    def linear_tiled(self, x, w_tiles, n_out: int, y, stream=None):
        """y = x @ w.T on the weight-streaming kernel, w given as its tiled copy (tile_weight):
        x [M, K], y [M, n_out] device bf16."""
        abi.call("gdn_linear_tiled", self.h, x.shape[0], n_out, x.shape[1], _ptr(x), x.stride(0), _ptr(w_tiles),
                 _ptr(y), y.stride(0), _stream(stream))

    def linear_q4(self, x, w_q4_tiles, n_out: int, y, stream=None):
        """y = x @ dequant(w).T, w an MLX 4-bit weight given as its tiled copy (tile_weight_q4)."""
        abi.call("gdn_linear_q4", self.h, x.shape[0], n_out, x.shape[1], _ptr(x), x.stride(0), _ptr(w_q4_tiles),
                 _ptr(y), y.stride(0), _stream(stream))

    def mixer_step(self, layer: int, w: MixerWeights, x, y, slot_ids, cu_seqlens, n_tokens: int, stream=None):
        """Whole mixer layer: y = out_proj(step(in_proj(x))); x, y [N, hidden] device bf16."""
        abi.call("gdn_mixer_step", self.h, layer, C.byref(w.c), _ptr(x), x.stride(0), _ptr(y), y.stride(0),
                 _ptr(slot_ids), _ptr(cu_seqlens), slot_ids.numel(), n_tokens, _stream(stream))

    def stack_step(self, ws, h, slot_ids, cu_seqlens, n_tokens: int, stream=None):
        """Residual GDN stack over all pool layers, in place on h [N, hidden] device bf16."""
        arr = (abi.GdnMixerWeightsC * len(ws))(*[w.c for w in ws])
        abi.call("gdn_stack_step", self.h, arr, _ptr(h), h.stride(0), _ptr(slot_ids), _ptr(cu_seqlens),
                 slot_ids.numel(), n_tokens, _stream(stream))

    def recurrence(self, layer: int, q, k, v, g, beta, y, slot_ids, cu_seqlens, n_tokens: int, stream=None):
        abi.call("gdn_recurrence", self.h, layer, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(slot_ids),
                 _ptr(cu_seqlens), slot_ids.numel(), n_tokens, _ptr(y), _stream(stream))
