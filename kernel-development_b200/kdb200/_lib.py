"""ctypes binding of libkdb200.so (the C ABI in include/kdb200.h).

The library is loaded from kernel-development_b200/lib/libkdb200.so.  There is no fallback: if the
library is missing or fails to load, every op raises RuntimeError naming the build command.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libkdb200.so"

KDB_OK = 0
KDB_ERR_INVALID_ARG = 1
KDB_ERR_UNSUPPORTED = 2
KDB_ERR_CUDA = 3
KDB_ERR_TIMEOUT = 4
KDB_ERR_WORKSPACE = 5
KDB_ERR_NO_DEVICE = 6
KDB_ERR_DEVICE_BOUNDS = 7

_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size = ctypes.c_size_t

# name -> (restype, argtypes); every symbol declared in include/kdb200.h
SIGNATURES: dict[str, tuple] = {
    "kdb_abi_version": (_c_int, []),
    "kdb_strerror": (ctypes.c_char_p, [_c_int]),
    "kdb_last_cuda_error": (_c_int, []),
    "kdb_status_read": (_c_int, [ctypes.POINTER(ctypes.c_uint32), _c_int, _c_vp]),
    "kdb_selftest_wait_timeout": (_c_int, [ctypes.c_uint64, _c_vp]),
    "kdb_proj_bf16": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp]),
    "kdb_proj_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "kdb_proj_bf16_ws": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "kdb_proj_tile_shape": (_c_int, [_c_i64, _c_i64, ctypes.POINTER(ctypes.c_int32)]),
    "kdb_set_sm_budget": (_c_int, [ctypes.c_int32]),
    "kdb_moe_w4a16_workspace_bytes": (_c_size, [_c_i64] * 6),
    "kdb_moe_w4a16_forward": (_c_int, [_c_vp] * 9 + [_c_i64] * 6 + [_c_vp, _c_size, _c_vp]),
    "kdb_attn_decode_workspace_bytes": (_c_size, [_c_i64] * 6),
    "kdb_attn_decode_fp8": (_c_int, [_c_vp] * 7 + [ctypes.c_float, _c_vp] + [_c_i64] * 8 + [_c_vp, _c_size, _c_vp]),
    "kdb_sm_budget": (_c_int, []),
    "kdb_proj_split_f32": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "kdb_proj_f32w_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "kdb_proj_f32w": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "kdb_proj_bf16_cfg": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_vp]),
    "kdb_moe_workspace_bytes": (_c_size, [_c_i64] * 7),
    "kdb_moe_pack_gate_up": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp]),
    "kdb_moe_route": (_c_int, [_c_vp] * 6 + [_c_i64] * 4 + [_c_vp]),
    "kdb_moe_plan_workspace_bytes": (_c_size, [_c_i64] * 3),
    "kdb_moe_plan": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_size,
                              _c_vp]),
    "kdb_moe_plan_noalloc": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),
    "kdb_moe_prepare_router": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "kdb_moe_router_approx": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp]),
    "kdb_moe_route_fast_workspace_bytes": (_c_size, [_c_i64, _c_i64]),
    "kdb_moe_route_fast": (_c_int, [_c_vp] * 7 + [_c_i64] * 4 + [_c_vp, _c_size, _c_vp]),
    "kdb_moe_gather_rows": (_c_int, [_c_vp, _c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp]),
    "kdb_moe_expert_gate_up": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp]),
    "kdb_moe_expert_down": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp,
                                     _c_vp]),
    "kdb_moe_combine": (_c_int, [_c_vp] * 5 + [_c_i64] * 3 + [_c_vp]),
    "kdb_moe_expert_down_combine_workspace_bytes": (_c_size, [_c_i64, _c_i64]),
    "kdb_moe_expert_down_combine": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64] + [_c_vp] * 8
                                    + [_c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "kdb_moe_ep_regroup_workspace_bytes": (_c_size, [_c_i64, _c_i64]),
    "kdb_moe_ep_regroup": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp,
                                    _c_size, _c_vp]),
    "kdb_moe_forward": (_c_int, [_c_vp] * 12 + [_c_i64] * 7 + [_c_vp, _c_size, _c_vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class KdbError(RuntimeError):
    """A libkdb200 entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int, detail: str = ""):
        self.code = code
        super().__init__(f"{fn} failed: {strerror(code)} (code {code}){detail}")


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises RuntimeError when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python kernel-development_b200/build.py` "
                    "(there is no CPU fallback for these ops)")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def strerror(code: int) -> str:
    try:
        return lib().kdb_strerror(int(code)).decode()
    except Exception:  # noqa: BLE001 - used while formatting another error
        return "unknown"


def check(fn: str, code: int) -> None:
    if code != KDB_OK:
        detail = ""
        if code == KDB_ERR_CUDA:
            detail = f"; cudaError {lib().kdb_last_cuda_error()}"
        raise KdbError(fn, code, detail)


def status_read(stream: int = 0, clear: bool = True) -> tuple[int, int, int, int]:
    """(first error code, site, block, reports) of the current device's status word (synchronises)."""
    out = (ctypes.c_uint32 * 4)()
    check("kdb_status_read", lib().kdb_status_read(out, 1 if clear else 0, _c_vp(stream)))
    return tuple(int(v) for v in out)  # type: ignore[return-value]
