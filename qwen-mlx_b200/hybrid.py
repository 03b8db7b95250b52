"""Host-side mirror of the hybrid decoder's other two layer kinds, over libgdn_b200.so (include/gdn_hybrid.h).

  * AttnConfig / KVCache / attn_step: the full-attention mixer body between its projections
    (Qwen35Attention::forward_with_cache, src/models/qwen3_5.rs:377-459) for a continuously batched
    step: sequences address a slot of a device-resident KV cache, as the GDN states address the
    state pool, instead of the executor stacking and zero-padding per-sequence caches
    (src/scheduler/mlx_executor.rs:57-86).
  * MoeConfig / MoeWeights / moe_route / moe_step: SparseMoeBlock::forward (qwen3_5.rs:262-302)
    with the checkpoint's MLX 4-bit experts and shared expert.

The q/k/v/o projections of the attention layer are plain library GEMMs around attn_step, as the GDN
mixer's default projections are.  Every call runs the library's kernels; nothing here computes on
the host.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import abi
from .gdn import _check_dev, _ptr, _stream, bf16_to_device


@dataclass(frozen=True)
class AttnConfig:
    """Attention fields of Qwen35Config (qwen3_5.rs:30-45); defaults are Qwen3.5-35B-A3B's."""
    n_heads: int = 16
    n_kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64            # head_dim * partial_rotary_factor (0.25)
    rope_theta: float = 10_000_000.0
    rms_norm_eps: float = 1e-6
    max_ctx: int = 4096

    def c(self) -> abi.GdnAttnConfigC:
        return abi.GdnAttnConfigC(self.n_heads, self.n_kv_heads, self.head_dim, self.rotary_dim, self.rope_theta,
                                  self.rms_norm_eps, self.max_ctx)

    def as_dict(self) -> dict:
        return dict(n_heads=self.n_heads, n_kv_heads=self.n_kv_heads, head_dim=self.head_dim,
                    rotary_dim=self.rotary_dim, rope_theta=self.rope_theta, rms_norm_eps=self.rms_norm_eps)


class KVCache:
    """Slot-indexed KV cache of one attention layer: k, v bf16 [n_slots][n_kv_heads][max_ctx][head_dim]."""

    def __init__(self, cfg: AttnConfig, n_slots: int, device):
        shape = (n_slots, cfg.n_kv_heads, cfg.max_ctx, cfg.head_dim)
        self.cfg = cfg
        self.n_slots = n_slots
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)


def attn_workspace_bytes(cfg: AttnConfig, n_tokens: int, max_kv_len: int) -> int:
    out = C.c_int64(0)
    abi.call("gdn_attn_workspace_bytes", C.byref(cfg.c()), int(n_tokens), int(max_kv_len), C.byref(out))
    return int(out.value)


def attn_step(cache: KVCache, q_full, k_in, v_in, q_norm_w, k_norm_w, slot_ids, cu_seqlens, positions, out=None,
              workspace=None, stream=None):
    """gdn_attn_step.  q_full [N][2*nh*hd], k_in / v_in [N][nkv*hd], q_norm_w / k_norm_w [hd]: bf16 CUDA tensors.
    slot_ids, cu_seqlens, positions: host integer sequences.  Returns out [N][nh*hd] bf16."""
    cfg = cache.cfg
    slots = np.ascontiguousarray(slot_ids, np.int32)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    pos = np.ascontiguousarray(positions, np.int32)
    n_seq, n_tok = len(slots), int(q_full.shape[0])
    for t, name in ((q_full, "q_full"), (k_in, "k_in"), (v_in, "v_in"), (q_norm_w, "q_norm_w"),
                    (k_norm_w, "k_norm_w")):
        _check_dev(t, name)
    if out is None:
        out = torch.empty((n_tok, cfg.n_heads * cfg.head_dim), dtype=torch.bfloat16, device=q_full.device)
    lens = np.diff(cu) if len(cu) > 1 else np.zeros(0, np.int32)
    max_kv = int((pos + lens).max()) if n_seq else 0
    need = attn_workspace_bytes(cfg, n_tok, max_kv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q_full.device)
    abi.call("gdn_attn_step", C.byref(cfg.c()), _ptr(q_full), _ptr(k_in), _ptr(v_in), _ptr(q_norm_w), _ptr(k_norm_w),
             _ptr(cache.k), _ptr(cache.v), cache.n_slots, slots.ctypes.data_as(C.c_void_p),
             cu.ctypes.data_as(C.c_void_p), pos.ctypes.data_as(C.c_void_p), n_seq, n_tok, _ptr(out), _ptr(workspace),
             int(workspace.numel()), _stream(stream))
    return out


# ------------------------------------------------------------------ MoE

@dataclass(frozen=True)
class MoeConfig:
    """MoE fields of Qwen35Config (qwen3_5.rs:55-63); defaults are Qwen3.5-35B-A3B's."""
    hidden: int = 2048
    n_experts: int = 256
    top_k: int = 8
    moe_inter: int = 512
    shared_inter: int = 512
    norm_topk_prob: bool = True

    def c(self) -> abi.GdnMoeConfigC:
        return abi.GdnMoeConfigC(self.hidden, self.n_experts, self.top_k, self.moe_inter, self.shared_inter,
                                 1 if self.norm_topk_prob else 0)

    def as_dict(self) -> dict:
        return dict(hidden=self.hidden, n_experts=self.n_experts, top_k=self.top_k, moe_inter=self.moe_inter,
                    shared_inter=self.shared_inter, norm_topk_prob=self.norm_topk_prob)


def _q4_dev(m: dict, device):
    q = torch.from_numpy(np.ascontiguousarray(m["q"], np.uint32).view(np.int32)).to(device)
    return q, bf16_to_device(m["scales"], device), bf16_to_device(m["biases"], device)


class MoeWeights:
    """Device copies of one MoE block: router [E][H] bf16, the stacked 4-bit experts (gate / up
    [E*moe_inter][H], down [E*H][moe_inter]), the 4-bit shared expert and the shared-expert gate [H] bf16.
    `w` is a dict of numpy arrays in the checkpoint's layout (q uint32 words, scales / biases bf16)."""

    def __init__(self, w: dict, device):
        self.router = bf16_to_device(w["router"], device) if w.get("router") is not None else None
        self.shared_gate = bf16_to_device(w["shared_gate"], device)
        self.mats = {k: _q4_dev(w[k], device) for k in ("gate", "up", "down", "sh_gate", "sh_up", "sh_down")}
        mc = {k: abi.GdnQ4MatrixC(*(_ptr(t) for t in v)) for k, v in self.mats.items()}
        self.c = abi.GdnMoeWeightsC(_ptr(self.router), mc["gate"], mc["up"], mc["down"], mc["sh_gate"], mc["sh_up"],
                                    mc["sh_down"], _ptr(self.shared_gate))


def moe_workspace_bytes(cfg: MoeConfig, n_tokens: int) -> int:
    out = C.c_int64(0)
    abi.call("gdn_moe_workspace_bytes", C.byref(cfg.c()), int(n_tokens), C.byref(out))
    return int(out.value)


def moe_route(cfg: MoeConfig, w: MoeWeights, x, want_logits: bool = False, stream=None):
    """gdn_moe_route: (ids int32 [N][k], weights bf16 [N][k], logits bf16 [N][E] or None)."""
    _check_dev(x, "x")
    n = int(x.shape[0])
    ids = torch.empty((n, cfg.top_k), dtype=torch.int32, device=x.device)
    wts = torch.empty((n, cfg.top_k), dtype=torch.bfloat16, device=x.device)
    logits = torch.empty((n, cfg.n_experts), dtype=torch.bfloat16, device=x.device) if want_logits else None
    abi.call("gdn_moe_route", C.byref(cfg.c()), C.byref(w.c), _ptr(x), n, _ptr(logits), _ptr(ids), _ptr(wts),
             _stream(stream))
    return ids, wts, logits


def moe_step(cfg: MoeConfig, w: MoeWeights, x, route=None, out=None, workspace=None, stream=None):
    """gdn_moe_step: the MoE block on x [N][hidden] bf16.  route: optional (ids, weights) device tensors."""
    _check_dev(x, "x")
    n = int(x.shape[0])
    if out is None:
        out = torch.empty((n, cfg.hidden), dtype=torch.bfloat16, device=x.device)
    need = moe_workspace_bytes(cfg, n)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    ids, wts = route if route is not None else (None, None)
    abi.call("gdn_moe_step", C.byref(cfg.c()), C.byref(w.c), _ptr(x), n, _ptr(ids), _ptr(wts), _ptr(out),
             _ptr(workspace), int(workspace.numel()), _stream(stream))
    return out
