"""CPU tests of the C ABI library: it loads, exports every declared symbol, and its
host-side argument checks and routing validation behave (no GPU work is issued)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def declared_functions():
    text = "".join(h.read_text() for h in sorted(INCLUDE.glob("*.h")))
    return sorted(set(re.findall(r"GDN_API\s+[\w\s\*]*?\b(gdn_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "gdn_layer_step" in names and "gdn_gated_delta_kernel" in names
    assert "gdn_sched_plan" in names and "gdn_pack_step" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol(abi):
    L = abi.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert set(declared_functions()) <= set(abi.SIGNATURES)


def test_version(abi):
    assert b"sm_100a" in abi.lib().gdn_version()


def _tables(slots, lens):
    s = np.ascontiguousarray(slots, np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return s, cu


def _validate(abi, n_slots, s, cu, n_tokens=None):
    n_tokens = int(cu[-1]) if n_tokens is None else n_tokens
    return abi.lib().gdn_validate_tables(n_slots, s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                                         len(s), n_tokens)


def test_validate_tables_accepts_ragged_batch(abi):
    s, cu = _tables([5, 0, 7, 2], [1, 3, 0, 5])
    assert _validate(abi, 8, s, cu) == abi.GDN_OK
    assert abi.last_error() == ""


@pytest.mark.parametrize("slots,lens,n_tokens,code", [
    ([5, 0, 5], [1, 1, 1], None, 3),      # duplicate slot
    ([8], [1], None, 3),                  # slot out of range
    ([-1], [1], None, 3),                 # negative slot
    ([0, 1], [2, 1], 4, 4),               # cu_seqlens[n] != n_tokens
])
def test_validate_tables_rejects(abi, slots, lens, n_tokens, code):
    s, cu = _tables(slots, lens)
    assert _validate(abi, 8, s, cu, n_tokens) == code
    assert abi.last_error() != ""


def test_validate_tables_rejects_decreasing_and_nonzero_start(abi):
    s = np.array([0, 1], np.int32)
    cu = np.array([0, 3, 2], np.int32)
    assert _validate(abi, 8, s, cu, 2) == abi.GDN_E_BAD_SEQLENS
    cu = np.array([1, 2, 3], np.int32)
    assert _validate(abi, 8, s, cu, 3) == abi.GDN_E_BAD_SEQLENS


def test_validate_empty_batch(abi):
    s = np.zeros(0, np.int32)
    cu = np.zeros(1, np.int32)
    assert _validate(abi, 4, s, cu, 0) == abi.GDN_OK
    assert _validate(abi, 4, s, cu, 3) == abi.GDN_E_BAD_SEQLENS


def test_pool_create_rejects_bad_config_before_touching_a_device(abi):
    L = abi.lib()
    h = C.c_void_p()
    assert L.gdn_pool_create(0, None, 4, C.byref(h)) == abi.GDN_E_INVALID
    bad = abi.GdnConfigC(2048, 16, 32, 64, 128, 4, 30, 1e-6)    # dk = 64 not specialised
    assert L.gdn_pool_create(0, C.byref(bad), 4, C.byref(h)) == abi.GDN_E_UNSUPPORTED
    bad = abi.GdnConfigC(2048, 16, 24, 128, 128, 4, 30, 1e-6)   # Hv not a multiple of Hk
    assert L.gdn_pool_create(0, C.byref(bad), 4, C.byref(h)) == abi.GDN_E_INVALID
    bad = abi.GdnConfigC(2048, 16, 32, 128, 128, 3, 30, 1e-6)   # conv kernel 3
    assert L.gdn_pool_create(0, C.byref(bad), 4, C.byref(h)) == abi.GDN_E_UNSUPPORTED
    assert not h.value


def test_null_pool_calls_fail_cleanly(abi):
    L = abi.lib()
    assert L.gdn_pool_destroy(None) == abi.GDN_OK
    assert L.gdn_layer_step(None, 0, None, None, None, None, 0, 0, None) == abi.GDN_E_INVALID
    assert L.gdn_recurrence(None, 0, None, None, None, None, None, None, None, 0, 0, None, None) == abi.GDN_E_INVALID
    f = C.c_int32()
    assert L.gdn_pool_check(None, C.byref(f), 0) == abi.GDN_E_INVALID
    assert L.gdn_gated_delta_kernel(None, None, None, None, None, None, 1, 1, 16, 32, 128, 128, None, None,
                                    None) == abi.GDN_E_INVALID


def test_gated_delta_kernel_rejects_unsupported_head_dim(abi):
    L = abi.lib()
    p = C.c_void_p(16)   # never dereferenced: argument checks come first
    assert L.gdn_gated_delta_kernel(p, p, p, p, p, p, 1, 1, 16, 32, 64, 128, p, p, None) == abi.GDN_E_UNSUPPORTED
    assert L.gdn_gated_delta_kernel(p, p, p, p, p, p, 1, 1, 16, 24, 128, 128, p, p, None) == abi.GDN_E_INVALID
