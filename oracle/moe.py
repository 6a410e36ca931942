"""Oracle for the fused MoE layer (test infrastructure; see oracle/__init__.py).

Layer math (bf16 activations and expert weights, fp32 router and accumulation):
  logits = x · Wrᵀ (+ bias)                       fp32, fixed-order fp64 dot rounded once (routing.c)
  ids    = top-k(logits), descending, ties -> lower expert index
  w      = softmax(logits)[ids] / sum(softmax(logits)[ids])       fp32 (renormalised top-k)
  for each routed (t, j):  e = ids[t, j]
      g, u = x[t] · Wg[e]ᵀ, x[t] · Wu[e]ᵀ          fp32 from bf16 operands
      h    = bf16( silu(g) * u )                    the GPU keeps the intermediate in bf16
      y[t] += w[t, j] * (h · Wd[e]ᵀ)                fp32
  shared expert (weight 1) adds the same SwiGLU expert on every token.
  Y = bf16(y)

Structure mirrors the reference engine's stages: routing plan (okc-challenge/engines/x3_h.cu:346-385),
gate_up + SwiGLU epilogue (sc_h.cu:322-340), down projection and weighted combine (sc_h.cu:341-381).
The reference's post-expert RMS normalisation and NVFP4 weights belong to its w4a16 problem, not to
this bf16 layer.
"""
from __future__ import annotations

import numpy as np
import torch

from . import routing_lib

# Output tolerances against this fp32 oracle (max-abs AND relative Frobenius); routing ids and the
# permutation must match exactly; routing weights to fp32 rounding.
MAX_ABS_TOL = 2e-2
REL_FRO_TOL = 1e-2
WEIGHT_RTOL = 1e-5


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def router_logits(x: torch.Tensor, router: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [T, E] logits in the fixed fp64 order of routing.c."""
    xb = np.ascontiguousarray(x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))
    wr = np.ascontiguousarray(router.detach().cpu().float().numpy())
    b = None if bias is None else np.ascontiguousarray(bias.detach().cpu().float().numpy())
    T, H = xb.shape
    E = wr.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    routing_lib().oracle_router_logits(_ptr(xb), _ptr(wr), None if b is None else _ptr(b), T, H, E, _ptr(out))
    return torch.from_numpy(out)


def topk(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(ids int32 [T, k], values fp32 [T, k]): descending, ties -> lower expert index."""
    lg = np.ascontiguousarray(logits.detach().cpu().float().numpy())
    T, E = lg.shape
    ids = np.empty((T, k), dtype=np.int32)
    vals = np.empty((T, k), dtype=np.float32)
    routing_lib().oracle_topk(_ptr(lg), T, E, k, _ptr(ids), _ptr(vals))
    return torch.from_numpy(ids), torch.from_numpy(vals)


def renorm_weights(logits: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """softmax over all experts, gathered at ids, renormalised over the k picks (fp32)."""
    p = torch.softmax(logits.float(), dim=-1)
    pk = p.gather(1, ids.long())
    return pk / pk.sum(dim=-1, keepdim=True)


def route(x, router, bias, k):
    """(logits, ids, weights) of the layer's router."""
    lg = router_logits(x, router, bias)
    ids, _ = topk(lg, k)
    return lg, ids, renorm_weights(lg, ids)


def permute(ids: torch.Tensor, e: int) -> dict:
    """Stable (expert, token) permutation plan of routing.c: counts, offsets, perm_slot, slot_pos."""
    a = np.ascontiguousarray(ids.detach().cpu().numpy().astype(np.int32))
    T, k = a.shape
    counts = np.empty(e, dtype=np.int32)
    offsets = np.empty(e + 1, dtype=np.int32)
    perm_slot = np.empty(T * k, dtype=np.int32)
    slot_pos = np.empty(T * k, dtype=np.int32)
    rc = routing_lib().oracle_permute(_ptr(a), T, k, e, _ptr(counts), _ptr(offsets), _ptr(perm_slot), _ptr(slot_pos))
    if rc != 0:
        raise ValueError("expert id out of range")
    return {"counts": torch.from_numpy(counts), "offsets": torch.from_numpy(offsets),
            "perm_slot": torch.from_numpy(perm_slot), "slot_pos": torch.from_numpy(slot_pos)}


def _expert(xe: torch.Tensor, gu: torch.Tensor, dn: torch.Tensor) -> torch.Tensor:
    """One SwiGLU expert on fp32 rows xe: down(bf16(silu(gate) * up)) in fp32."""
    i = gu.shape[0] // 2
    guf = gu.float()
    g = xe @ guf[:i].T
    u = xe @ guf[i:].T
    h = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
    return h @ dn.float().T


def moe_ref(x: torch.Tensor, weights: dict, k: int, route_out=None) -> dict:
    """Full layer on the CPU.  Returns {"y": bf16[T, H], "y32": fp32[T, H], "ids", "w", "logits"}.
    Experts are converted to fp32 one at a time (a full fp32 copy of a large layer does not fit)."""
    x = x.detach().cpu()
    router = weights["router"]
    bias = weights.get("router_bias")
    lg, ids, w = route_out if route_out is not None else route(x, router, bias, k)
    gu, dn = weights["w_gate_up"], weights["w_down"]
    E = gu.shape[0]
    T, H = x.shape
    xf = x.float()
    y = torch.zeros((T, H), dtype=torch.float32)
    flat_ids = ids.reshape(-1).long()
    flat_w = w.reshape(-1)
    tok = torch.arange(T).repeat_interleave(k)
    for e in range(E):
        sel = (flat_ids == e).nonzero().flatten()
        if sel.numel() == 0:
            continue
        rows = tok[sel]
        ye = _expert(xf[rows], gu[e].cpu(), dn[e].cpu())
        y.index_add_(0, rows, ye * flat_w[sel, None])
    sgu, sdn = weights.get("shared_gate_up"), weights.get("shared_down")
    if sgu is not None:
        for s in range(sgu.shape[0]):
            y += _expert(xf, sgu[s].cpu(), sdn[s].cpu())
    return {"y": y.to(torch.bfloat16), "y32": y, "ids": ids, "w": w, "logits": lg}


def torch_fp32_logits(x: torch.Tensor, router: torch.Tensor, bias=None) -> torch.Tensor:
    """The plain fp32 torch router (x.float() @ Wr.T + b): used to show that the fixed-order logits
    route identically to it except where its own logits tie within fp32 rounding."""
    lg = x.detach().cpu().float() @ router.detach().cpu().float().T
    if bias is not None:
        lg = lg + bias.detach().cpu().float()
    return lg


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """max-abs, relative Frobenius and worst-row (token) relative L2 error of `out` against fp32 `ref`."""
    o, r = out.detach().cpu().float(), ref.detach().cpu().float()
    d = o - r
    rows = d.norm(dim=-1) / r.norm(dim=-1).clamp_min(1e-30) if r.dim() == 2 else d.abs()
    return {"max_abs": float(d.abs().max()) if d.numel() else 0.0,
            "rel_fro": float(d.norm() / r.norm().clamp_min(1e-30)),
            "worst_row": float(rows.max()) if rows.numel() else 0.0,
            "nonfinite": int((~torch.isfinite(o)).sum())}


def check(out: tuple, ref: dict) -> tuple[bool, str]:
    """(ok, message) for a layer output (y, topk_w, topk_ids) against moe_ref's result."""
    if not isinstance(out, (tuple, list)) or len(out) != 3:
        return False, "expected (y, topk_weights, topk_ids)"
    y, w, ids = out
    if tuple(y.shape) != tuple(ref["y"].shape) or tuple(ids.shape) != tuple(ref["ids"].shape):
        return False, f"shape mismatch: y {tuple(y.shape)} ids {tuple(ids.shape)}"
    id_bad = int((ids.detach().cpu().to(torch.int32) != ref["ids"].to(torch.int32)).sum())
    wc = compare(w, ref["w"])
    yc = compare(y, ref["y32"])
    ok = (id_bad == 0 and yc["nonfinite"] == 0 and yc["max_abs"] <= MAX_ABS_TOL and yc["rel_fro"] <= REL_FRO_TOL
          and wc["max_abs"] <= WEIGHT_RTOL * 10)
    msg = (f"relative L2 error {yc['rel_fro']:.3e} (worst row {yc['worst_row']:.3e}) max-abs {yc['max_abs']:.3e}; "
           f"routing ids mismatched {id_bad}; weights max-abs {wc['max_abs']:.3e} "
           f"[bound {REL_FRO_TOL}: max-abs <= {MAX_ABS_TOL}, ids exact]")
    return ok, msg
