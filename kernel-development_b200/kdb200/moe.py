"""Fused MoE layer as PyTorch custom ops over libkdb200.

Forward signature follows kdev's problem-adapter contract (src/kdev/adapters/okc.py:501-537):
`prepare(weights) -> state` once (untimed; packs gate/up rows), then `kernel_fn(data, state)` with
data = {"x": bf16[T, H], "config": {...}} returning (y bf16[T, H], topk_w fp32[T, k],
topk_ids int32[T, k]) — routing ids at output index 2 as in the reference's routing problems
(src/kdev/adapters/okc_problems/muse_prefill_layer.toml:148).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_vp = ctypes.c_void_p


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> int | None:
    return None if t is None else t.data_ptr()


def _need(name: str, t: torch.Tensor, dtype: torch.dtype, dim: int) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _same_device(dev: torch.device, **tensors: Optional[torch.Tensor]) -> None:
    for name, t in tensors.items():
        if t is not None and t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev} (the kernels read every operand there)")


def _check_groups(a: torch.Tensor, width: int, groups: int, offsets: Optional[torch.Tensor],
                  mtile_start: Optional[torch.Tensor]) -> None:
    """Rows a [R, width] grouped by offsets [groups + 1] (+ the m-tile prefix, same length) on a's device."""
    if a.shape[1] != width:
        raise ValueError(f"rows are {a.shape[1]} wide, the weights expect {width}")
    for name, t in (("offsets", offsets), ("mtile_start", mtile_start)):
        if t is not None:
            _need(name, t, torch.int32, 1)
            if t.numel() != groups + 1:
                raise ValueError(f"{name} must have groups + 1 = {groups + 1} entries")
    _same_device(a.device, offsets=offsets, mtile_start=mtile_start)


def pack_gate_up(w_gate_up: torch.Tensor) -> torch.Tensor:
    """[E, 2I, H] (gate rows then up rows) -> the packed layout the gate_up GEMM reads."""
    _need("w_gate_up", w_gate_up, torch.bfloat16, 3)
    e, two_i, h = w_gate_up.shape
    out = torch.empty_like(w_gate_up)
    with torch.cuda.device(w_gate_up.device):
        rc = _lib.lib().kdb_moe_pack_gate_up(w_gate_up.data_ptr(), out.data_ptr(), e, two_i // 2, h,
                                              _vp(_stream(w_gate_up.device)))
    _lib.check("kdb_moe_pack_gate_up", rc)
    return out


def route(x: torch.Tensor, router: torch.Tensor, bias: Optional[torch.Tensor], k: int):
    """(logits fp32 [T, E], topk_w fp32 [T, k], topk_ids int32 [T, k]) of the router stage."""
    _need("x", x, torch.bfloat16, 2)
    _need("router", router, torch.float32, 2)
    if bias is not None:
        _need("bias", bias, torch.float32, 1)
    _same_device(x.device, router=router, bias=bias)
    t, h = x.shape
    e = router.shape[0]
    if router.shape[1] != h or (bias is not None and tuple(bias.shape) != (e,)):
        raise ValueError(f"router must be [E, {h}] and bias [E]")
    logits = torch.empty((t, e), dtype=torch.float32, device=x.device)
    w = torch.empty((t, k), dtype=torch.float32, device=x.device)
    ids = torch.empty((t, k), dtype=torch.int32, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_route(x.data_ptr(), router.data_ptr(), _ptr(bias), logits.data_ptr(), w.data_ptr(),
                                      ids.data_ptr(), t, h, e, k, _vp(_stream(x.device)))
    _lib.check("kdb_moe_route", rc)
    return logits, w, ids


def plan(ids: torch.Tensor, topk_w: torch.Tensor, e: int) -> dict:
    """Permutation plan: counts [E], offsets [E+1], perm_slot [T*k], slot_pos [T*k] (int32)."""
    _need("topk_ids", ids, torch.int32, 2)
    _need("topk_w", topk_w, torch.float32, 2)
    if topk_w.shape != ids.shape:
        raise ValueError("topk_ids and topk_w must have the same shape")
    t, k = ids.shape
    dev = ids.device
    _same_device(dev, topk_w=topk_w)
    counts = torch.empty(e, dtype=torch.int32, device=dev)
    offsets = torch.empty(e + 1, dtype=torch.int32, device=dev)
    perm_slot = torch.empty(t * k, dtype=torch.int32, device=dev)
    slot_pos = torch.empty(t * k, dtype=torch.int32, device=dev)
    nbytes = _lib.lib().kdb_moe_plan_workspace_bytes(t, e, k)
    ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().kdb_moe_plan(ids.data_ptr(), topk_w.data_ptr(), t, e, k, counts.data_ptr(), offsets.data_ptr(),
                                     perm_slot.data_ptr(), slot_pos.data_ptr(), ws.data_ptr(), ws.numel(),
                                     _vp(_stream(dev)))
    _lib.check("kdb_moe_plan", rc)
    return {"counts": counts, "offsets": offsets, "perm_slot": perm_slot, "slot_pos": slot_pos}


def prepare_router(router: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(router_split bf16 [E, 2H], router_norms fp32 [E]) for the tensor-core routing path."""
    _need("router", router, torch.float32, 2)
    e, h = router.shape
    split = torch.empty((e, 2 * h), dtype=torch.bfloat16, device=router.device)
    norms = torch.empty(e, dtype=torch.float32, device=router.device)
    with torch.cuda.device(router.device):
        rc = _lib.lib().kdb_moe_prepare_router(router.data_ptr(), split.data_ptr(), norms.data_ptr(), e, h,
                                               _vp(_stream(router.device)))
    _lib.check("kdb_moe_prepare_router", rc)
    return split, norms


def router_approx(x: torch.Tensor, split: torch.Tensor) -> torch.Tensor:
    """fp32 [T, E] tensor-core pre-pass logits x · [W_hi | W_mid]ᵀ (without bias)."""
    _need("x", x, torch.bfloat16, 2)
    _need("split", split, torch.bfloat16, 2)
    _same_device(x.device, split=split)
    t, h = x.shape
    e = split.shape[0]
    if split.shape[1] != 2 * h:
        raise ValueError(f"split must be [E, {2 * h}] (prepare_router)")
    out = torch.empty((t, e), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_router_approx(x.data_ptr(), split.data_ptr(), out.data_ptr(), t, h, e,
                                              _vp(_stream(x.device)))
    _lib.check("kdb_moe_router_approx", rc)
    return out


def route_fast(x: torch.Tensor, router: torch.Tensor, bias: Optional[torch.Tensor], split: torch.Tensor,
               norms: torch.Tensor, k: int):
    """(topk_w, topk_ids) of the tensor-core routing path (identical to route()'s)."""
    _need("x", x, torch.bfloat16, 2)
    _need("router", router, torch.float32, 2)
    _need("split", split, torch.bfloat16, 2)
    _need("norms", norms, torch.float32, 1)
    if bias is not None:
        _need("bias", bias, torch.float32, 1)
    _same_device(x.device, router=router, bias=bias, split=split, norms=norms)
    t, h = x.shape
    e = router.shape[0]
    if (router.shape[1] != h or tuple(split.shape) != (e, 2 * h) or tuple(norms.shape) != (e,)
            or (bias is not None and tuple(bias.shape) != (e,))):
        raise ValueError(f"router [E, {h}], split [E, {2 * h}], norms [E] and bias [E] expected")
    w = torch.empty((t, k), dtype=torch.float32, device=x.device)
    ids = torch.empty((t, k), dtype=torch.int32, device=x.device)
    nbytes = int(_lib.lib().kdb_moe_route_fast_workspace_bytes(t, e))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_route_fast(x.data_ptr(), router.data_ptr(), _ptr(bias), split.data_ptr(),
                                           norms.data_ptr(), w.data_ptr(), ids.data_ptr(), t, h, e, k, ws.data_ptr(),
                                           ws.numel(), _vp(_stream(x.device)))
    _lib.check("kdb_moe_route_fast", rc)
    return w, ids


def workspace_bytes(t: int, h: int, e: int, i: int, k: int, shared: int = 0, shared_i: int = 0) -> int:
    n = int(_lib.lib().kdb_moe_workspace_bytes(t, h, e, i, k, shared, shared_i))
    if n == 0 and t > 0:
        raise ValueError(f"unsupported MoE shape t={t} h={h} e={e} i={i} k={k} shared={shared}/{shared_i}")
    return n


@torch.library.custom_op("kdb200::moe", mutates_args=())
def moe(x: torch.Tensor, router: torch.Tensor, router_bias: Optional[torch.Tensor], router_split: Optional[torch.Tensor],
        router_norms: Optional[torch.Tensor], w_gate_up_packed: torch.Tensor, w_down: torch.Tensor,
        shared_gate_up_packed: Optional[torch.Tensor], shared_down: Optional[torch.Tensor],
        k: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The fused MoE layer; returns (y bf16[T, H], topk_w fp32[T, k], topk_ids int32[T, k])."""
    _need("x", x, torch.bfloat16, 2)
    _need("router", router, torch.float32, 2)
    _need("w_gate_up_packed", w_gate_up_packed, torch.bfloat16, 3)
    _need("w_down", w_down, torch.bfloat16, 3)
    t, h = x.shape
    e, two_i, h2 = w_gate_up_packed.shape
    i = two_i // 2
    if h2 != h or tuple(w_down.shape) != (e, h, i) or tuple(router.shape) != (e, h):
        raise ValueError("inconsistent MoE weight shapes")
    shared, shared_i = 0, 0
    if shared_gate_up_packed is not None:
        _need("shared_gate_up_packed", shared_gate_up_packed, torch.bfloat16, 3)
        _need("shared_down", shared_down, torch.bfloat16, 3)
        shared, shared_i = shared_gate_up_packed.shape[0], shared_gate_up_packed.shape[1] // 2
    if router_bias is not None:
        _need("router_bias", router_bias, torch.float32, 1)
        if tuple(router_bias.shape) != (e,):
            raise ValueError(f"router_bias must be [{e}]")
    if (router_split is None) != (router_norms is None):
        raise ValueError("router_split and router_norms come together (prepare_router)")
    if router_split is not None:
        _need("router_split", router_split, torch.bfloat16, 2)
        _need("router_norms", router_norms, torch.float32, 1)
        if tuple(router_split.shape) != (e, 2 * h) or tuple(router_norms.shape) != (e,):
            raise ValueError(f"router_split must be [{e}, {2 * h}] and router_norms [{e}]")
    if shared_gate_up_packed is not None and tuple(shared_down.shape) != (shared, h, shared_i):
        raise ValueError(f"shared_down must be [{shared}, {h}, {shared_i}]")
    dev = x.device
    _same_device(dev, router=router, router_bias=router_bias, router_split=router_split, router_norms=router_norms,
                 w_gate_up_packed=w_gate_up_packed, w_down=w_down, shared_gate_up_packed=shared_gate_up_packed,
                 shared_down=shared_down)
    y = torch.empty((t, h), dtype=torch.bfloat16, device=dev)
    w = torch.empty((t, k), dtype=torch.float32, device=dev)
    ids = torch.empty((t, k), dtype=torch.int32, device=dev)
    nbytes = workspace_bytes(t, h, e, i, k, shared, shared_i)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().kdb_moe_forward(
            x.data_ptr(), router.data_ptr(), _ptr(router_bias), _ptr(router_split), _ptr(router_norms),
            w_gate_up_packed.data_ptr(), w_down.data_ptr(),
            _ptr(shared_gate_up_packed), _ptr(shared_down), y.data_ptr(), w.data_ptr(), ids.data_ptr(),
            t, h, e, i, k, shared, shared_i, ws.data_ptr(), ws.numel(), _vp(_stream(dev)))
    _lib.check("kdb_moe_forward", rc)
    return y, w, ids


@moe.register_fake
def _moe_fake(x, router, router_bias, router_split, router_norms, w_gate_up_packed, w_down, shared_gate_up_packed,
              shared_down, k):
    t, h = x.shape
    return (x.new_empty((t, h)), x.new_empty((t, k), dtype=torch.float32), x.new_empty((t, k), dtype=torch.int32))


def prepare(weights: dict, k: int) -> dict:
    """Untimed state for kernel_fn: packed gate/up weights; other weights referenced as given
    (the caller's tensors are not modified, and every value is kept bit-exact)."""
    dev = weights["w_gate_up"].device
    if not weights["w_gate_up"].is_cuda:
        raise ValueError("MoE weights must be on a CUDA device")
    sgu = weights.get("shared_gate_up")
    bias = weights.get("router_bias")
    router = weights["router"].contiguous()
    split, norms = prepare_router(router) if router.shape[1] % 64 == 0 else (None, None)
    return {
        "k": int(k),
        "router": router,
        "router_split": split,
        "router_norms": norms,
        "router_bias": None if bias is None else bias.to(dev).contiguous(),
        "w_gate_up_packed": pack_gate_up(weights["w_gate_up"].contiguous()),
        "w_down": weights["w_down"].contiguous(),
        "shared_gate_up_packed": None if sgu is None else pack_gate_up(sgu.contiguous()),
        "shared_down": None if sgu is None else weights["shared_down"].contiguous(),
    }


def forward(x: torch.Tensor, state: dict):
    return moe(x, state["router"], state["router_bias"], state.get("router_split"), state.get("router_norms"),
               state["w_gate_up_packed"], state["w_down"], state["shared_gate_up_packed"], state["shared_down"],
               state["k"])


# ------------------------------------------------------------------------------------ stage entry points
def gather_rows(x: torch.Tensor, index: torch.Tensor, div: int = 1, rows: Optional[int] = None) -> torch.Tensor:
    """out[r] = x[index[r] // div] (bf16 rows)."""
    _need("x", x, torch.bfloat16, 2)
    _need("index", index, torch.int32, 1)
    _same_device(x.device, index=index)
    n = index.numel() if rows is None else int(rows)
    if not 0 <= n <= index.numel():
        raise ValueError(f"rows ({n}) must be within the index's {index.numel()} entries")
    out = torch.empty((n, x.shape[1]), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_gather_rows(x.data_ptr(), index.data_ptr(), div, out.data_ptr(), n, x.shape[1],
                                            x.shape[0], _vp(_stream(x.device)))
    _lib.check("kdb_moe_gather_rows", rc)
    return out


def expert_gate_up(a: torch.Tensor, w_packed: torch.Tensor, offsets: Optional[torch.Tensor] = None,
                   mtile_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Grouped gate_up + SwiGLU: a bf16 [R, H] (rows grouped as offsets say) -> bf16 [R, I]."""
    _need("a", a, torch.bfloat16, 2)
    _need("w_packed", w_packed, torch.bfloat16, 3)
    groups, two_i, h = w_packed.shape
    _check_groups(a, h, groups, offsets, mtile_start)
    out = torch.empty((a.shape[0], two_i // 2), dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        rc = _lib.lib().kdb_moe_expert_gate_up(a.data_ptr(), a.shape[0], w_packed.data_ptr(), groups, two_i // 2, h,
                                               _ptr(offsets), _ptr(mtile_start), out.data_ptr(), _vp(_stream(a.device)))
    _lib.check("kdb_moe_expert_gate_up", rc)
    return out


def expert_down(a: torch.Tensor, w_down: torch.Tensor, offsets: Optional[torch.Tensor] = None,
                mtile_start: Optional[torch.Tensor] = None, row_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Grouped down projection: a bf16 [R, I] -> bf16 [R, H] (rows scaled by row_scale when given)."""
    _need("a", a, torch.bfloat16, 2)
    _need("w_down", w_down, torch.bfloat16, 3)
    groups, h, i = w_down.shape
    _check_groups(a, i, groups, offsets, mtile_start)
    if row_scale is not None:
        _need("row_scale", row_scale, torch.float32, 1)
        _same_device(a.device, row_scale=row_scale)
        if row_scale.numel() != a.shape[0]:
            raise ValueError(f"row_scale must have one entry per row ({a.shape[0]})")
    out = torch.empty((a.shape[0], h), dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        rc = _lib.lib().kdb_moe_expert_down(a.data_ptr(), a.shape[0], w_down.data_ptr(), groups, i, h, _ptr(offsets),
                                            _ptr(mtile_start), _ptr(row_scale), out.data_ptr(), _vp(_stream(a.device)))
    _lib.check("kdb_moe_expert_down", rc)
    return out


def expert_down_combine(a: torch.Tensor, w_down: torch.Tensor, offsets: torch.Tensor, mtile_start: torch.Tensor,
                        row_scale: torch.Tensor, perm_slot: torch.Tensor, slot_pos: torch.Tensor, t: int, k: int,
                        shared_rows: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Grouped down with the combine merged into its epilogue (one launch): returns (per-slot rows bf16
    [R, H], y bf16 [t, H]); y equals combine(rows, slot_pos, t, k, shared_rows=shared_rows) bitwise."""
    _need("a", a, torch.bfloat16, 2)
    _need("w_down", w_down, torch.bfloat16, 3)
    groups, h, i = w_down.shape
    _check_groups(a, i, groups, offsets, mtile_start)
    for name, v in (("row_scale", row_scale),):
        _need(name, v, torch.float32, 1)
    _need("perm_slot", perm_slot, torch.int32, 1)
    _need("slot_pos", slot_pos, torch.int32, 1)
    if row_scale.numel() != a.shape[0] or perm_slot.numel() != a.shape[0] or slot_pos.numel() != t * k:
        raise ValueError("row_scale and perm_slot need one entry per row, slot_pos t * k entries")
    if shared_rows is not None:
        _need("shared_rows", shared_rows, torch.bfloat16, 2)
        if tuple(shared_rows.shape) != (t, h):
            raise ValueError(f"shared_rows must be [{t}, {h}]")
    _same_device(a.device, row_scale=row_scale, perm_slot=perm_slot, slot_pos=slot_pos, shared_rows=shared_rows)
    rows = torch.empty((a.shape[0], h), dtype=torch.bfloat16, device=a.device)
    y = torch.empty((t, h), dtype=torch.bfloat16, device=a.device)
    nbytes = int(_lib.lib().kdb_moe_expert_down_combine_workspace_bytes(t, h))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=a.device)
    with torch.cuda.device(a.device):
        rc = _lib.lib().kdb_moe_expert_down_combine(
            a.data_ptr(), a.shape[0], w_down.data_ptr(), groups, i, h, offsets.data_ptr(), mtile_start.data_ptr(),
            row_scale.data_ptr(), perm_slot.data_ptr(), slot_pos.data_ptr(), _ptr(shared_rows), rows.data_ptr(),
            y.data_ptr(), t, k, ws.data_ptr(), ws.numel(), _vp(_stream(a.device)))
    _lib.check("kdb_moe_expert_down_combine", rc)
    return rows, y


def combine(rows: torch.Tensor, slot_pos: torch.Tensor, t: int, k: int, slot_w: Optional[torch.Tensor] = None,
            shared_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[t] = sum_j (slot_w or 1) * rows[slot_pos[t*k + j]] (+ shared_rows[t]) in fp32, bf16 out."""
    _need("slot_pos", slot_pos, torch.int32, 1)
    if rows.dim() == 2:
        _need("rows", rows, torch.bfloat16, 2)
    elif shared_rows is None:
        raise ValueError("rows must be bf16 [R, H] unless shared_rows gives H")
    if slot_pos.numel() != t * k:
        raise ValueError(f"slot_pos must have t * k = {t * k} entries")
    if slot_w is not None:
        if slot_w.dtype != torch.float32 or slot_w.numel() != t * k or not slot_w.is_contiguous():
            raise ValueError(f"slot_w must be contiguous fp32 with t * k = {t * k} entries")
    if shared_rows is not None:
        _need("shared_rows", shared_rows, torch.bfloat16, 2)
    h = rows.shape[1] if rows.dim() == 2 else shared_rows.shape[1]
    if shared_rows is not None and tuple(shared_rows.shape) != (t, h):
        raise ValueError(f"shared_rows must be [{t}, {h}]")
    _same_device(slot_pos.device, rows=rows, slot_w=slot_w, shared_rows=shared_rows)
    y = torch.empty((t, h), dtype=torch.bfloat16, device=slot_pos.device)
    with torch.cuda.device(slot_pos.device):
        rc = _lib.lib().kdb_moe_combine(rows.data_ptr(), slot_pos.data_ptr(), _ptr(slot_w), _ptr(shared_rows),
                                        y.data_ptr(), t, h, k, _vp(_stream(slot_pos.device)))
    _lib.check("kdb_moe_combine", rc)
    return y


def ep_regroup(counts: torch.Tensor, rows_in: Optional[torch.Tensor], to_expert_major: bool,
               rows_out: Optional[torch.Tensor] = None):
    """Block transpose between source-major (s, e) and expert-major rows for counts int32 [P, Er];
    returns (rows_out, offsets [Er + 1], mtile_start [Er + 1])."""
    _need("counts", counts, torch.int32, 2)
    if rows_in is not None:
        _need("rows_in", rows_in, torch.bfloat16, 2)
        if rows_out is not None:
            _need("rows_out", rows_out, torch.bfloat16, 2)
            if rows_out.shape != rows_in.shape:
                raise ValueError("rows_out must have rows_in's shape")
    _same_device(counts.device, rows_in=rows_in, rows_out=rows_out)
    p, er = counts.shape
    dev = counts.device
    offsets = torch.empty(er + 1, dtype=torch.int32, device=dev)
    mtile = torch.empty(er + 1, dtype=torch.int32, device=dev)
    ws = torch.empty(max(int(_lib.lib().kdb_moe_ep_regroup_workspace_bytes(p, er)), 256), dtype=torch.uint8,
                     device=dev)
    if rows_in is not None and rows_out is None:
        rows_out = torch.empty_like(rows_in)
    h = rows_in.shape[1] if rows_in is not None else 8
    with torch.cuda.device(dev):
        rc = _lib.lib().kdb_moe_ep_regroup(counts.data_ptr(), p, er, 1 if to_expert_major else 0, _ptr(rows_in),
                                           _ptr(rows_out), h, offsets.data_ptr(), mtile.data_ptr(), ws.data_ptr(),
                                           ws.numel(), _vp(_stream(dev)))
    _lib.check("kdb_moe_ep_regroup", rc)
    return rows_out, offsets, mtile
