"""CPU tests of the C ABI: the library loads, exports every entry point include/kdb200.h declares,
and rejects bad arguments before touching the device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from kdb200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kdb200.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(kdb_[a-z0-9_]+)\s*\(", text))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("kdb_proj_bf16", "kdb_moe_forward", "kdb_moe_route", "kdb_moe_plan", "kdb_status_read"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(_declared()):
        assert hasattr(lib, name), f"{name} declared in include/kdb200.h but not exported"


def test_python_binding_covers_header():
    assert _declared() <= set(_lib.SIGNATURES), sorted(_declared() - set(_lib.SIGNATURES))


def test_abi_version_and_strerror(lib):
    assert lib.kdb_abi_version() == 2
    assert lib.kdb_strerror(0) == b"ok"
    assert b"timed out" in lib.kdb_strerror(_lib.KDB_ERR_TIMEOUT)
    assert lib.kdb_strerror(999) == b"unknown status"


def test_proj_argument_checks_without_device(lib):
    vp = ctypes.c_void_p
    # negative size, ldy < n, K not a multiple of 8, null pointers: all rejected on the host
    assert lib.kdb_proj_bf16(vp(16), vp(16), vp(16), -1, 8, 8, 8, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16(vp(16), vp(16), vp(16), 4, 8, 8, 4, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16(vp(16), vp(16), vp(16), 4, 8, 12, 8, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16(None, vp(16), vp(16), 4, 8, 8, 8, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16(vp(17), vp(16), vp(16), 4, 8, 8, 8, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16_cfg(vp(16), vp(16), vp(16), 4, 8, 8, 8, 96, 0, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_bf16_cfg(vp(16), vp(16), vp(16), 4, 8, 8, 8, 128, 1, None) == _lib.KDB_ERR_INVALID_ARG
    # empty problems are no-ops
    assert lib.kdb_proj_bf16(None, None, None, 0, 8, 8, 8, None) == 0
    assert lib.kdb_proj_bf16(None, None, None, 8, 0, 8, 8, None) == 0


def test_moe_workspace_and_shape_checks(lib):
    assert lib.kdb_moe_workspace_bytes(64, 4096, 64, 1024, 8, 0, 0) > 0
    # prefill: 8192 x 7168, 256 experts, top-8, shared expert: per-slot rows dominate
    big = lib.kdb_moe_workspace_bytes(8192, 7168, 256, 2048, 8, 1, 2048)
    assert 1.0e9 < big < 2.0e9
    assert lib.kdb_moe_workspace_bytes(64, 4096, 64, 1000, 8, 0, 0) == 0      # i % 128 != 0
    assert lib.kdb_moe_workspace_bytes(64, 4100, 64, 1024, 8, 0, 0) == 0      # h % 8 != 0
    assert lib.kdb_moe_workspace_bytes(64, 4096, 4, 1024, 8, 0, 0) == 0       # k > e
    assert lib.kdb_moe_workspace_bytes(64, 4096, 2048, 1024, 8, 0, 0) == 0    # e > 1024
    vp = ctypes.c_void_p
    rc = lib.kdb_moe_forward(*([vp(256)] * 12), 64, 4096, 64, 1024, 8, 0, 0, vp(256), 16, None)
    assert rc == _lib.KDB_ERR_WORKSPACE
    rc = lib.kdb_moe_route(vp(16), vp(16), None, vp(16), vp(16), vp(16), 4, 64, 8, 9, None)
    assert rc == _lib.KDB_ERR_INVALID_ARG
    rc = lib.kdb_moe_pack_gate_up(vp(16), vp(16), 2, 100, 64, None)
    assert rc == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_moe_plan_workspace_bytes(100, 16, 4) > 0


def test_w4a16_host_checks(lib):
    # one ep8 rank of the NVFP4 layer: 32 local of 256 experts, H = I = 4096, top-8
    assert lib.kdb_moe_w4a16_workspace_bytes(256, 4096, 4096, 32, 256, 8) > 0
    assert lib.kdb_moe_w4a16_workspace_bytes(256, 4000, 4096, 32, 256, 8) == 0   # H % 256 != 0
    assert lib.kdb_moe_w4a16_workspace_bytes(256, 4096, 4000, 32, 256, 8) == 0   # I % 128 != 0
    assert lib.kdb_moe_w4a16_workspace_bytes(256, 4096, 4096, 300, 256, 8) == 0  # local > total experts
    vp = ctypes.c_void_p
    ptrs = [vp(256)] * 9          # x, ids, tw, w13 blocks, gs13, w2 blocks, gs2, pw1, y
    shape = (16, 4096, 4096, 32, 256, 8)
    need = lib.kdb_moe_w4a16_workspace_bytes(*shape)
    # no tokens: nothing to do, whatever the pointers
    assert lib.kdb_moe_w4a16_forward(*([None] * 9), 0, 4096, 4096, 32, 256, 8, None, 0, None) == 0
    # null, misaligned, too small a workspace: rejected before any launch
    assert lib.kdb_moe_w4a16_forward(*([None] + ptrs[1:]), *shape, vp(256), need, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_moe_w4a16_forward(*([vp(264)] + ptrs[1:]), *shape, vp(256), need, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_moe_w4a16_forward(*ptrs, *shape, vp(256), need - 1, None) == _lib.KDB_ERR_WORKSPACE
    assert lib.kdb_moe_w4a16_forward(*ptrs, *shape, vp(384), need, None) == _lib.KDB_ERR_INVALID_ARG  # 256-B alignment
    assert lib.kdb_moe_w4a16_forward(*ptrs, 16, 4096, 4000, 32, 256, 8, vp(256), need, None) == _lib.KDB_ERR_UNSUPPORTED


def test_f32w_projection_host_checks(lib):
    vp = ctypes.c_void_p
    assert lib.kdb_proj_split_f32(None, None, 0, 7168, None) == 0
    assert lib.kdb_proj_split_f32(None, vp(16), 256, 7168, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_f32w(None, None, None, 0, 256, 7168, None, 0, None) == 0
    assert lib.kdb_proj_f32w(vp(16), vp(16), None, 4, 256, 7168, None, 0, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_f32w(vp(16), vp(16), vp(16), 4, 256, 7100, None, 0, None) == _lib.KDB_ERR_UNSUPPORTED
    assert lib.kdb_proj_f32w(vp(17), vp(16), vp(16), 4, 256, 7168, None, 0, None) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_proj_f32w_workspace_bytes(200, 256, 7168) == 0     # above 128 rows: no K split
    assert lib.kdb_proj_f32w_workspace_bytes(0, 256, 7168) == 0


def test_sm_budget_round_trip(lib):
    old = lib.kdb_set_sm_budget(16)
    try:
        assert lib.kdb_sm_budget() == 16
        assert lib.kdb_set_sm_budget(-5) == 16    # negative clears the budget
        assert lib.kdb_sm_budget() == 0
    finally:
        lib.kdb_set_sm_budget(old)
    assert lib.kdb_sm_budget() == old


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(RuntimeError, match="not built"):
        _lib.lib()
