"""Oracle for the bf16 projection (test infrastructure; see oracle/__init__.py).

Math of the `muse_bf16_proj` problem (src/kdev/adapters/okc_problems/muse_bf16_proj.toml:1-8):
Y = X · Wᵀ with bf16 operands, fp32 accumulation and a bf16 result.
"""
from __future__ import annotations

import torch

# Tolerances of the projection check: max-abs and relative Frobenius error against this
# fp32 reference (the bf16 rounding of Y alone gives a relative error near 2^-9 / sqrt(3)).  The max-abs
# bound is 2e-2 for outputs of unit scale (the benchmark distributions: X ~ N(0, 1), W ~ N(0, 1/K) give
# rms(Y) ~ 1) and grows with rms(Y) above that: for heavy-tailed inputs (the reference's "outliers"
# distribution, rms(Y) ~ 8) the bf16 rounding of the largest outputs alone is half a unit in the last
# place of |Y| ~ 32, i.e. 0.06.
MAX_ABS_TOL = 2e-2
REL_FRO_TOL = 1e-2


def max_abs_bound(ref: torch.Tensor) -> float:
    """MAX_ABS_TOL * max(1, rms(ref))."""
    r = ref.detach().cpu().float()
    rms = float(r.pow(2).mean().sqrt()) if r.numel() else 0.0
    return MAX_ABS_TOL * max(1.0, rms)


def proj_ref(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """fp32 [M, N] = x.float() @ w.float().T on the CPU."""
    return x.detach().cpu().float() @ w.detach().cpu().float().T


# fp32-weight (router) layer: the hi+mid split keeps each weight to 2^-16 and accumulation is fp32, so
# the output is checked far tighter than the bf16 layers.
ROUTER_REL_FRO_TOL = 1e-4
ROUTER_MAX_ABS_TOL = 1e-3
PROBE_REL_TOL = 1e-3   # probe rows (one nonzero power-of-two input) exact to 0.1% (muse_bf16_proj.toml:376)


def proj_ref_f32w(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """fp32 [M, N] = x · wᵀ with fp32 weights, accumulated in fp64 on the CPU (the router layer)."""
    return (x.detach().cpu().double() @ w.detach().cpu().double().T).float()


def check_f32w(out: torch.Tensor, ref: torch.Tensor) -> tuple[bool, str]:
    """(ok, message) for the fp32-output router layer."""
    if tuple(out.shape) != tuple(ref.shape) or out.dtype != torch.float32:
        return False, f"expected fp32 {tuple(ref.shape)}, got {out.dtype} {tuple(out.shape)}"
    c = compare(out, ref)
    ok = c["nonfinite"] == 0 and c["max_abs"] <= ROUTER_MAX_ABS_TOL and c["rel_fro"] <= ROUTER_REL_FRO_TOL
    msg = (f"relative L2 error {c['rel_fro']:.3e} (worst row {c['worst_row']:.3e}) max-abs {c['max_abs']:.3e} "
           f"[bound {ROUTER_REL_FRO_TOL}: max-abs <= {ROUTER_MAX_ABS_TOL}]")
    return ok, msg


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """max-abs, relative Frobenius and worst-row relative L2 error of `out` against fp32 `ref`."""
    o = out.detach().cpu().float()
    r = ref.detach().cpu().float()
    d = o - r
    fro = float(d.norm() / r.norm().clamp_min(1e-30))
    rows = d.norm(dim=-1) / r.norm(dim=-1).clamp_min(1e-30) if r.dim() == 2 else d.abs()
    return {
        "max_abs": float(d.abs().max()) if d.numel() else 0.0,
        "rel_fro": fro,
        "worst_row": float(rows.max()) if rows.numel() else 0.0,
        "nonfinite": int((~torch.isfinite(o)).sum()),
    }


def check(out: torch.Tensor, ref: torch.Tensor) -> tuple[bool, str]:
    """(ok, message) in the wording kdev's parse_check_message reads (src/kdev/adapters/okc.py:231-247)."""
    if tuple(out.shape) != tuple(ref.shape):
        return False, f"shape {tuple(out.shape)} != expected {tuple(ref.shape)}"
    c = compare(out, ref)
    mab = max_abs_bound(ref)
    ok = c["nonfinite"] == 0 and c["max_abs"] <= mab and c["rel_fro"] <= REL_FRO_TOL
    msg = (f"relative L2 error {c['rel_fro']:.3e} (worst row {c['worst_row']:.3e}) max-abs {c['max_abs']:.3e} "
           f"[bound {REL_FRO_TOL}: max-abs <= {mab:.3g}]")
    return ok, msg
