"""ctypes declarations of include/gdn.h, include/gdn_host.h and include/gdn_hybrid.h for libgdn_b200.so.

The library is the product; this module only binds it.  Loading fails loudly
when the library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libgdn_b200.so"

GDN_OK = 0
GDN_E_INVALID = 1
GDN_E_UNSUPPORTED = 2
GDN_E_BAD_SLOT = 3
GDN_E_BAD_SEQLENS = 4
GDN_E_CUDA = 5
GDN_E_NOMEM = 6
GDN_E_DEVICE = 7

GDN_ENTRY_DECODE = 0
GDN_ENTRY_PREFILL_FIRST = 1
GDN_ENTRY_PREFILL_CONT = 2
GDN_STEP_TABLES_STABLE = 1

GDN_FINISH_EOS = 0
GDN_FINISH_MAX_TOKENS = 1

# Every function declared in include/gdn.h, with (restype, argtypes).
_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_int = C.c_int


class GdnConfigC(C.Structure):
    _fields_ = [("hidden", _i32), ("n_k_heads", _i32), ("n_v_heads", _i32), ("head_k_dim", _i32),
                ("head_v_dim", _i32), ("conv_kernel", _i32), ("n_layers", _i32), ("rms_norm_eps", C.c_float)]


class GdnLayerWeightsC(C.Structure):
    _fields_ = [("conv_w", _vp), ("A_log", _vp), ("dt_bias", _vp), ("norm_w", _vp), ("dt_bias_bf16", _i32)]


class GdnStepIOC(C.Structure):
    _fields_ = [("qkv", _vp), ("ld_qkv", _i64), ("z", _vp), ("ld_z", _i64), ("ab", _vp), ("ld_ab", _i64),
                ("out", _vp), ("ld_out", _i64)]


class GdnMixerWeightsC(C.Structure):
    _fields_ = [("step", GdnLayerWeightsC), ("w_in", _vp), ("w_out", _vp), ("pre_norm_w", _vp),
                ("w_in_tiles", _vp), ("w_out_tiles", _vp), ("w_in_q4", _vp), ("w_out_q4", _vp)]


class GdnStepEntryC(C.Structure):
    _fields_ = [("seq_id", C.c_uint64), ("slot", _i32), ("n_tokens", _i32), ("kind", _i32), ("pos", _i32)]


class GdnSchedConfigC(C.Structure):
    _fields_ = [("n_shards", _i32), ("slots_per_shard", _i32), ("max_batch", _i32), ("prefill_budget", _i32),
                ("prefill_chunk", _i32)]


class GdnSchedStatsC(C.Structure):
    _fields_ = [("total_requests", C.c_uint64), ("tokens_generated", C.c_uint64), ("iterations", C.c_uint64),
                ("active", _i32), ("waiting", _i32), ("prefilling", _i32), ("free_slots", _i32)]


class GdnAttnConfigC(C.Structure):
    _fields_ = [("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32), ("rotary_dim", _i32),
                ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("max_ctx", _i32)]


class GdnMoeConfigC(C.Structure):
    _fields_ = [("hidden", _i32), ("n_experts", _i32), ("top_k", _i32), ("moe_inter", _i32), ("shared_inter", _i32),
                ("norm_topk_prob", _i32)]


class GdnQ4MatrixC(C.Structure):
    _fields_ = [("q", _vp), ("scales", _vp), ("biases", _vp)]


class GdnMoeWeightsC(C.Structure):
    _fields_ = [("router", _vp), ("gate", GdnQ4MatrixC), ("up", GdnQ4MatrixC), ("down", GdnQ4MatrixC),
                ("sh_gate", GdnQ4MatrixC), ("sh_up", GdnQ4MatrixC), ("sh_down", GdnQ4MatrixC), ("shared_gate", _vp)]


SIGNATURES = {
    "gdn_last_error": (C.c_char_p, []),
    "gdn_version": (C.c_char_p, []),
    "gdn_pool_create": (_int, [_int, C.POINTER(GdnConfigC), _i32, C.POINTER(_vp)]),
    "gdn_pool_destroy": (_int, [_vp]),
    "gdn_pool_reserve_tokens": (_int, [_vp, _i32]),
    "gdn_pool_layer_state": (_int, [_vp, _i32, C.POINTER(_vp), C.POINTER(_vp)]),
    "gdn_pool_bytes": (_int, [_vp, C.POINTER(C.c_size_t)]),
    "gdn_slot_reset": (_int, [_vp, _vp, _i32, _vp]),
    "gdn_slot_export": (_int, [_vp, _i32, _i32, _vp, _vp]),
    "gdn_slot_import": (_int, [_vp, _i32, _i32, _vp, _vp]),
    "gdn_validate_batch": (_int, [_vp, _vp, _vp, _i32, _i32]),
    "gdn_validate_tables": (_int, [_i32, _vp, _vp, _i32, _i32]),
    "gdn_pool_check": (_int, [_vp, C.POINTER(_i32), _int]),
    "gdn_layer_step": (_int, [_vp, _i32, C.POINTER(GdnLayerWeightsC), C.POINTER(GdnStepIOC), _vp, _vp, _i32, _i32,
                              _vp]),
    "gdn_layer_step_ex": (_int, [_vp, _i32, C.POINTER(GdnLayerWeightsC), C.POINTER(GdnStepIOC), _vp, _vp, _i32,
                                 _i32, C.c_uint32, _vp]),
    "gdn_linear": (_int, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _vp, _i64, _vp]),
    "gdn_weight_tile_bytes": (_i64, [_i32, _i32]),
    "gdn_weight_tile": (_int, [_i32, _i32, _vp, _vp, _vp]),
    "gdn_weight_tile_q4_bytes": (_i64, [_i32, _i32]),
    "gdn_weight_tile_q4": (_int, [_i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "gdn_linear_tiled": (_int, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _vp, _i64, _vp]),
    "gdn_linear_q4": (_int, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _vp, _i64, _vp]),
    "gdn_mixer_step": (_int, [_vp, _i32, C.POINTER(GdnMixerWeightsC), _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32,
                              _vp]),
    "gdn_stack_step": (_int, [_vp, C.POINTER(GdnMixerWeightsC), _vp, _i64, _vp, _vp, _i32, _i32, _vp]),
    "gdn_recurrence": (_int, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp]),
    "gdn_gated_delta_kernel": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                                      _vp]),
    "gdn_beta_g": (_int, [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "gdn_beta_g_ex": (_int, [_vp, _i64, _i32, _i32, _vp, _vp, _i32, _vp, _vp, _vp]),
    "gdn_layer_step_noalloc": (_int, [C.POINTER(GdnConfigC), _i32, _vp, _vp, C.POINTER(GdnLayerWeightsC),
                                      C.POINTER(GdnStepIOC), _vp, _vp, _i32, _i32, _vp]),
    "gdn_noalloc_check": (_int, [C.POINTER(_i32), _int]),
    "gdn_set_decode_kernel": (_int, [_int]),
    "gdn_test_set_wait_fault": (_int, [_i32, _i64]),
    # include/gdn_host.h
    "gdn_pack_step": (_int, [C.POINTER(GdnStepEntryC), _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "gdn_sched_create": (_int, [C.POINTER(GdnSchedConfigC), C.POINTER(_vp)]),
    "gdn_sched_destroy": (_int, [_vp]),
    "gdn_sched_enqueue": (_int, [_vp, _i32, _i32, C.POINTER(C.c_uint64)]),
    "gdn_sched_plan": (_int, [_vp, C.POINTER(GdnStepEntryC), _i32, C.POINTER(_i32)]),
    "gdn_sched_complete": (_int, [_vp, _vp]),
    "gdn_sched_drain_finished": (_int, [_vp, C.POINTER(C.c_uint64), C.POINTER(_i32), _i32, C.POINTER(_i32)]),
    "gdn_sched_stats_get": (_int, [_vp, C.POINTER(GdnSchedStatsC)]),
    "gdn_sched_active_ids": (_int, [_vp, C.POINTER(C.c_uint64), _i32, C.POINTER(_i32)]),
    "gdn_sched_free_slots": (_int, [_vp, _i32, C.POINTER(_i32)]),
    # include/gdn_hybrid.h
    "gdn_attn_workspace_bytes": (_int, [C.POINTER(GdnAttnConfigC), _i32, _i32, C.POINTER(_i64)]),
    "gdn_attn_step": (_int, [C.POINTER(GdnAttnConfigC), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _i32,
                             _i32, _vp, _vp, _i64, _vp]),
    "gdn_moe_workspace_bytes": (_int, [C.POINTER(GdnMoeConfigC), _i32, C.POINTER(_i64)]),
    "gdn_moe_route": (_int, [C.POINTER(GdnMoeConfigC), C.POINTER(GdnMoeWeightsC), _vp, _i32, _vp, _vp, _vp, _vp]),
    "gdn_moe_step": (_int, [C.POINTER(GdnMoeConfigC), C.POINTER(GdnMoeWeightsC), _vp, _i32, _vp, _vp, _vp, _vp, _i64,
                            _vp]),
}


class GdnError(RuntimeError):
    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func} failed with code {code}: {msg}")
        self.code = code
        self.func = func


_lib = None


def lib():
    """Load libgdn_b200.so (raises if it is missing or lacks a declared symbol)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python qwen-mlx_b200/build.py` (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().gdn_last_error().decode()


def check(rc: int, func: str):
    if rc != GDN_OK:
        raise GdnError(rc, func, last_error())


def call(name: str, *args):
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc
