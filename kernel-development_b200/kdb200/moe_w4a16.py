"""NVFP4 w4a16 MoE layer of one expert-parallel rank as a PyTorch custom op over libkdb200
(kdb_moe_w4a16_forward): the reference's `muse_moe_w4a16` problem
(src/kdev/adapters/okc_problems/muse_moe_w4a16.toml), whose engines stream NVFP4 expert weights
(okc-challenge/engines/sc_h.cu:189-467).

prepare(weights) reorders the NVFP4 tensors losslessly so that every 128-row x 64-element block keeps its
codes and scales contiguous (one bulk copy each in the kernel); the weights stay NVFP4.
"""
from __future__ import annotations

import torch

from . import _lib


def _tile(codes: torch.Tensor, scales: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """codes uint8 [L, rows, K/2], scales e4m3 [L, rows, K/16] -> [L, rows/128, K/64, 128, 32] and
    [L, rows/128, K/64, 128, 4] (bytes)."""
    L, rows, half = codes.shape
    K = 2 * half
    if rows % 128 or K % 64:
        raise ValueError(f"NVFP4 tensor [{rows}, {K}] is not tileable (rows % 128, K % 64)")
    c = codes.contiguous().view(L, rows // 128, 128, K // 64, 32).permute(0, 1, 3, 2, 4).contiguous()
    s = scales.contiguous().view(torch.uint8).view(L, rows // 128, 128, K // 64, 4).permute(0, 1, 3, 2, 4)
    return c, s.contiguous()


def prepare(weights: dict, device: str | torch.device = "cuda") -> dict:
    """Untimed: tile the NVFP4 weights for the kernel (the caller's tensors are not modified)."""
    w13c, w13s = _tile(weights["w13"].to(device), weights["w13_scale"].to(device))
    w2c, w2s = _tile(weights["w2"].to(device), weights["w2_scale"].to(device))
    L, rows13, _ = weights["w13"].shape
    return {"w13_codes": w13c, "w13_scales": w13s, "w13_gscale": weights["w13_gscale"].to(device).float().contiguous(),
            "w2_codes": w2c, "w2_scales": w2s, "w2_gscale": weights["w2_gscale"].to(device).float().contiguous(),
            "local": L, "i": rows13 // 2, "h": weights["w2"].shape[1]}


@torch.library.custom_op("kdb200::moe_w4a16", mutates_args=())
def moe_w4a16(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, w13_codes: torch.Tensor,
              w13_scales: torch.Tensor, w13_gscale: torch.Tensor, w2_codes: torch.Tensor, w2_scales: torch.Tensor,
              w2_gscale: torch.Tensor, e_total: int) -> torch.Tensor:
    """y bf16 [T, H]: the rank's local routes (ids < local) through NVFP4 experts, RMS-normalised and
    weighted (kdb_moe_w4a16_forward)."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise TypeError("x must be a contiguous bf16 [T, H] CUDA tensor (there is no CPU path)")
    if topk_ids.dtype != torch.int32 or topk_w.dtype != torch.float32 or topk_ids.shape != topk_w.shape:
        raise TypeError("topk_ids int32 and topk_w fp32, both [T, k]")
    t, h = x.shape
    k = topk_ids.shape[1]
    local = w13_codes.shape[0]
    i = w13_codes.shape[1] * 128 // 2
    y = torch.empty((t, h), dtype=torch.bfloat16, device=x.device)
    nbytes = int(_lib.lib().kdb_moe_w4a16_workspace_bytes(t, h, i, local, e_total, k))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_w4a16_forward(
            x.data_ptr(), topk_ids.contiguous().data_ptr(), topk_w.contiguous().data_ptr(), w13_codes.data_ptr(),
            w13_scales.data_ptr(), w13_gscale.data_ptr(), w2_codes.data_ptr(), w2_scales.data_ptr(),
            w2_gscale.data_ptr(), y.data_ptr(), t, h, i, local, e_total, k, ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check("kdb_moe_w4a16_forward", rc)
    return y


@moe_w4a16.register_fake
def _moe_w4a16_fake(x, topk_ids, topk_w, w13_codes, w13_scales, w13_gscale, w2_codes, w2_scales, w2_gscale, e_total):
    return x.new_empty(x.shape)


def forward(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, state: dict, e_total: int) -> torch.Tensor:
    return moe_w4a16(x, topk_ids, topk_w, state["w13_codes"], state["w13_scales"], state["w13_gscale"],
                     state["w2_codes"], state["w2_scales"], state["w2_gscale"], int(e_total))
