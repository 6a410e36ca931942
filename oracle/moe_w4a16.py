"""Oracle for the NVFP4 w4a16 MoE layer (test infrastructure; see oracle/__init__.py).

The layer of one expert-parallel rank, as the reference's H200 engines compute it for its
`muse_moe_w4a16` problem (src/kdev/adapters/okc_problems/muse_moe_w4a16.toml): NVFP4 expert weights
(E2M1 codes, E4M3 scale per 16 elements, fp32 global scale), bf16 activations, fp32 accumulation, only the
routes to this rank's experts (ids < local) computed, and a post-expert RMS normalisation:

  for each local route (t, j), e = ids[t, j] < local:
      W13 = e2m1 * scale (exact in bf16); g, u = x[t] . W1[e]^T * gs13[e], x[t] . W3[e]^T * gs13[e]
      h   = bf16( silu(g) * u )                                   (sc_h.cu:322-340)
      y   = (h . W2[e]^T) * gs2[e] * pw1                           fp32, pw1 [H] a per-feature weight
                                                                   (sc_h.cu:51, 209, 346; x3_h.cu:110, 345, 529)
      out[t] += y * tw[t, j] * rsqrt(mean(y^2) + 1e-8)             y stays fp32 through the sum of squares
                                                                   (sc_h.cu:347-351, 380; x3_h.cu:530-535, 654-656)
  OUT = bf16(out)

The reference's problem package (reference.py, its NVFP4 layout and checks) is not in its tree, so the
weight layout here is the common NVFP4 one (codes [rows, cols/2] low nibble first, scales [rows, cols/16])
and parity with the reference is unpinned.
"""
from __future__ import annotations

import torch

from kdb200 import workloads as W

MAX_ABS_TOL = 2e-2
REL_FRO_TOL = 1e-2
RMS_EPS = 1e-8


def dequant_expert(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 e2m1 * e4m3 for one expert tensor (global scale not applied)."""
    return W.nvfp4_dequantize(codes, scales)


def w4a16_ref(x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, weights: dict, local: int) -> torch.Tensor:
    """fp32 [T, H] layer output (before the final bf16 rounding) on the CPU.  weights["pw1"] (fp32 [H]) is the
    engines' per-feature output weight; absent, it is 1."""
    x = x.detach().cpu()
    ids, tw = ids.detach().cpu(), tw.detach().cpu().float()
    T, H = x.shape
    out = torch.zeros((T, H), dtype=torch.float32)
    I = weights["w13"].shape[1] // 2
    xf = x.float()
    pw1 = weights.get("pw1")
    pw1 = torch.ones(H) if pw1 is None else pw1.detach().cpu().float()
    for e in range(local):
        rows = (ids == e).nonzero()
        if rows.numel() == 0:
            continue
        tok, slot = rows[:, 0], rows[:, 1]
        w13 = dequant_expert(weights["w13"][e], weights["w13_scale"][e])
        w2 = dequant_expert(weights["w2"][e], weights["w2_scale"][e])
        gs13, gs2 = float(weights["w13_gscale"][e]), float(weights["w2_gscale"][e])
        gu = (xf[tok] @ w13.T) * gs13
        g, u = gu[:, :I], gu[:, I:]
        h = (g / (1.0 + torch.exp(-g)) * u).to(torch.bfloat16).float()
        y = (h @ w2.T) * gs2 * pw1                           # fp32, as the engines keep it
        rms = torch.rsqrt((y * y).mean(dim=1, keepdim=True) + RMS_EPS)
        out.index_add_(0, tok, y * tw[tok, slot].unsqueeze(1) * rms)
    return out


def check(out: torch.Tensor, ref: torch.Tensor) -> tuple[bool, str]:
    o = out.detach().cpu().float()
    d = o - ref
    fro = float(d.norm() / ref.norm().clamp_min(1e-30))
    mx = float(d.abs().max()) if d.numel() else 0.0
    ok = bool(torch.isfinite(o).all()) and mx <= MAX_ABS_TOL and fro <= REL_FRO_TOL
    rows = d.norm(dim=-1) / ref.norm(dim=-1).clamp_min(1e-30)
    return ok, (f"relative L2 error {fro:.3e} (worst row {float(rows.max()) if rows.numel() else 0.0:.3e}) "
                f"max-abs {mx:.3e} [bound {REL_FRO_TOL}: max-abs <= {MAX_ABS_TOL}]")
