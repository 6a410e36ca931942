"""kdb_moe_plan_noalloc: the routing-plan entry point for callers that cannot allocate device memory.

Such callers (a runtime that reserves all device memory at start-up and binds this library over a C
FFI, or code that must not call cudaMalloc) pass only the plan's inputs and outputs; the entry point
uses a fixed scratch array inside the library instead of a workspace.  These tests call it through
the C ABI and require its outputs to equal those of kdb_moe_plan (the workspace entry point) exactly
— the plan is integer work, so the tolerance is zero — on two calls in a row, the second one smaller
than the first so that the shared array still holds the first call's contents.  They pass alone in a
fresh process and after the rest of the suite (this file sorts last)."""
from __future__ import annotations

import ctypes

import pytest
import torch

from kdb200 import _lib

pytestmark = pytest.mark.gpu

_vp = ctypes.c_void_p


def _routing(t: int, e: int, k: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ids = torch.rand((t, e), generator=g, device="cuda").argsort(dim=1)[:, :k].to(torch.int32).contiguous()
    w = torch.rand((t, k), generator=g, device="cuda").contiguous()
    return ids, w


def _outputs(t: int, e: int, k: int):
    dev = "cuda"
    return (torch.full((e,), -7, dtype=torch.int32, device=dev), torch.full((e + 1,), -7, dtype=torch.int32, device=dev),
            torch.full((t * k,), -7, dtype=torch.int32, device=dev), torch.full((t * k,), -7, dtype=torch.int32, device=dev))


def _plan_with_workspace(ids, w, e):
    t, k = ids.shape
    counts, offsets, perm_slot, slot_pos = _outputs(t, e, k)
    nbytes = _lib.lib().kdb_moe_plan_workspace_bytes(t, e, k)
    ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device="cuda")
    rc = _lib.lib().kdb_moe_plan(ids.data_ptr(), w.data_ptr(), t, e, k, counts.data_ptr(), offsets.data_ptr(),
                                 perm_slot.data_ptr(), slot_pos.data_ptr(), ws.data_ptr(), ws.numel(),
                                 _vp(torch.cuda.current_stream().cuda_stream))
    _lib.check("kdb_moe_plan", rc)
    return counts, offsets, perm_slot, slot_pos


def _plan_noalloc(ids, w, e):
    t, k = ids.shape
    counts, offsets, perm_slot, slot_pos = _outputs(t, e, k)
    rc = _lib.lib().kdb_moe_plan_noalloc(ids.data_ptr(), w.data_ptr(), t, e, k, counts.data_ptr(), offsets.data_ptr(),
                                         perm_slot.data_ptr(), slot_pos.data_ptr(),
                                         _vp(torch.cuda.current_stream().cuda_stream))
    _lib.check("kdb_moe_plan_noalloc", rc)
    return counts, offsets, perm_slot, slot_pos


def test_noalloc_plan_equals_workspace_plan_twice():
    names = ("counts", "offsets", "perm_slot", "slot_pos")
    for (t, e, k, seed) in [(3000, 64, 8, 1), (500, 128, 4, 2)]:
        ids, w = _routing(t, e, k, seed)
        want = _plan_with_workspace(ids, w, e)
        got = _plan_noalloc(ids, w, e)
        torch.cuda.synchronize()
        for name, a, b in zip(names, got, want):
            assert torch.equal(a, b), f"{name} differs at t={t} e={e} k={k}"
        assert int(got[1][-1]) == t * k


def test_noalloc_plan_rejects_sizes_beyond_its_array():
    ids, w = _routing(4, 8, 2, 3)
    lib = _lib.lib()
    # t * k above 131072 slots, e above 1024 experts: rejected before any launch
    rc = lib.kdb_moe_plan_noalloc(ids.data_ptr(), w.data_ptr(), 65537, 8, 2, _vp(16), _vp(16), _vp(16), _vp(16), None)
    assert rc == _lib.KDB_ERR_UNSUPPORTED
    rc = lib.kdb_moe_plan_noalloc(ids.data_ptr(), w.data_ptr(), 4, 1025, 2, _vp(16), _vp(16), _vp(16), _vp(16), None)
    assert rc == _lib.KDB_ERR_UNSUPPORTED
    # within the slot and expert limits but ceil(t / 256) * e = 256 * 1024 chunk cells > 65536
    rc = lib.kdb_moe_plan_noalloc(ids.data_ptr(), w.data_ptr(), 65536, 1024, 1, _vp(16), _vp(16), _vp(16), _vp(16),
                                  None)
    assert rc == _lib.KDB_ERR_UNSUPPORTED
    assert b"not supported" in lib.kdb_strerror(rc)
