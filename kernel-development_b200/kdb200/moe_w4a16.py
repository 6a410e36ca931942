"""NVFP4 w4a16 MoE layer of one expert-parallel rank as a PyTorch custom op over libkdb200
(kdb_moe_w4a16_forward): the reference's `muse_moe_w4a16` problem
(src/kdev/adapters/okc_problems/muse_moe_w4a16.toml), whose engines stream NVFP4 expert weights
(okc-challenge/engines/sc_h.cu:189-467).

prepare(weights) reorders the NVFP4 tensors losslessly into 9 KB blocks (both parts' codes and scales of
one weight tile and k chunk, chunks consecutive), which the kernel fetches two at a time with one bulk
copy; the weights stay NVFP4.
"""
from __future__ import annotations

import torch

from . import _lib


def _blocks(codes: torch.Tensor, scales: torch.Tensor, gate_up: bool) -> torch.Tensor:
    """NVFP4 codes uint8 [L, rows, K/2] + scales e4m3 [L, rows, K/16] -> uint8 blocks [L, F, K/64, 9216]:
    per weight tile f and 64-element k chunk, [part 0 codes (128 x 32 B) | part 1 codes | part 0 scales
    (128 x 4 B) | part 1 scales].  gate_up: rows [0, I) gate and [I, 2I) up, tile f = gate rows 128f.. and
    up rows I + 128f..; otherwise tile f = rows 256f.. as two 128-row parts."""
    L, rows, half = codes.shape
    K = 2 * half
    if K % 128 or rows % 256:
        raise ValueError(f"NVFP4 tensor [{rows}, {K}] is not tileable (rows % 256, K % 128)")
    KC = K // 64
    c = codes.contiguous()
    sc = scales.contiguous().view(torch.uint8)
    if gate_up:
        F = rows // 256
        c = c.view(L, 2, F, 128, KC, 32).permute(0, 2, 4, 1, 3, 5)          # [L, F, KC, part, 128, 32]
        sc = sc.view(L, 2, F, 128, KC, 4).permute(0, 2, 4, 1, 3, 5)
    else:
        F = rows // 256
        c = c.view(L, F, 2, 128, KC, 32).permute(0, 1, 4, 2, 3, 5)
        sc = sc.view(L, F, 2, 128, KC, 4).permute(0, 1, 4, 2, 3, 5)
    return torch.cat([c.reshape(L, F, KC, 2 * 4096), sc.reshape(L, F, KC, 2 * 512)], dim=-1).contiguous()


def prepare(weights: dict, device: str | torch.device = "cuda") -> dict:
    """Untimed: reorder the NVFP4 weights into the kernel's blocks (the caller's tensors are not modified)."""
    w13 = _blocks(weights["w13"].to(device), weights["w13_scale"].to(device), gate_up=True)
    w2 = _blocks(weights["w2"].to(device), weights["w2_scale"].to(device), gate_up=False)
    L, rows13, _ = weights["w13"].shape
    h = weights["w2"].shape[1]
    pw1 = weights.get("pw1")
    pw1 = torch.ones(h, dtype=torch.float32) if pw1 is None else pw1
    return {"w13_blocks": w13, "w13_gscale": weights["w13_gscale"].to(device).float().contiguous(),
            "w2_blocks": w2, "w2_gscale": weights["w2_gscale"].to(device).float().contiguous(),
            "pw1": pw1.to(device).float().contiguous(), "local": L, "i": rows13 // 2, "h": h}


def _check(x, topk_ids, topk_w, w13_blocks, w13_gscale, w2_blocks, w2_gscale, pw1, e_total):
    """Shapes, dtypes and devices of kdb200::moe_w4a16's arguments; returns (T, H, I, local, k).  The kernel
    receives raw pointers, so every tensor must be contiguous and on x's CUDA device."""
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be bf16 [T, H]")
    if topk_ids.dtype != torch.int32 or topk_w.dtype != torch.float32 or topk_ids.dim() != 2:
        raise TypeError("topk_ids must be int32 and topk_w fp32, both [T, k]")
    if w13_blocks.dtype != torch.uint8 or w2_blocks.dtype != torch.uint8 or w13_blocks.dim() != 4:
        raise TypeError("NVFP4 blocks must be uint8 [local, tiles, k chunks, 9216] (use moe_w4a16.prepare)")
    if w13_gscale.dtype != torch.float32 or w2_gscale.dtype != torch.float32:
        raise TypeError("global scales must be fp32 [local]")
    t, h = x.shape
    k = topk_ids.shape[1]
    local = w13_blocks.shape[0]
    i = w13_blocks.shape[1] * 128
    if topk_ids.shape != topk_w.shape or topk_ids.shape[0] != t:
        raise ValueError(f"topk_ids {tuple(topk_ids.shape)} and topk_w {tuple(topk_w.shape)} must be [{t}, k]")
    if tuple(w13_blocks.shape[2:]) != (h // 64, 9216) or tuple(w2_blocks.shape) != (local, h // 256, i // 64, 9216):
        raise ValueError("NVFP4 blocks do not match x's hidden size (use moe_w4a16.prepare)")
    if tuple(w13_gscale.shape) != (local,) or tuple(w2_gscale.shape) != (local,):
        raise ValueError(f"global scales must be [{local}]")
    if pw1.dtype != torch.float32 or tuple(pw1.shape) != (h,):
        raise ValueError(f"pw1 must be fp32 [{h}]")
    if not local <= e_total:
        raise ValueError(f"e_total ({e_total}) must be at least the number of local experts ({local})")
    tensors = (x, topk_ids, topk_w, w13_blocks, w13_gscale, w2_blocks, w2_gscale, pw1)
    if not x.is_cuda or any(a.device != x.device for a in tensors):
        raise ValueError("all tensors must be on one CUDA device (there is no CPU path)")
    if not all(a.is_contiguous() for a in tensors):
        raise ValueError("all tensors must be contiguous")
    return t, h, i, local, k


@torch.library.custom_op("kdb200::moe_w4a16", mutates_args=())
def moe_w4a16(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, w13_blocks: torch.Tensor,
              w13_gscale: torch.Tensor, w2_blocks: torch.Tensor, w2_gscale: torch.Tensor, pw1: torch.Tensor,
              e_total: int) -> torch.Tensor:
    """y bf16 [T, H]: the rank's local routes (ids < local) through NVFP4 experts, times the per-feature
    weight pw1, RMS-normalised and weighted (kdb_moe_w4a16_forward)."""
    t, h, i, local, k = _check(x, topk_ids, topk_w, w13_blocks, w13_gscale, w2_blocks, w2_gscale, pw1, e_total)
    y = torch.empty((t, h), dtype=torch.bfloat16, device=x.device)
    nbytes = int(_lib.lib().kdb_moe_w4a16_workspace_bytes(t, h, i, local, e_total, k))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.lib().kdb_moe_w4a16_forward(
            x.data_ptr(), topk_ids.data_ptr(), topk_w.data_ptr(), w13_blocks.data_ptr(),
            w13_gscale.data_ptr(), w2_blocks.data_ptr(), w2_gscale.data_ptr(), pw1.data_ptr(), y.data_ptr(), t, h, i,
            local, e_total,
            k, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check("kdb_moe_w4a16_forward", rc)
    return y


@moe_w4a16.register_fake
def _moe_w4a16_fake(x, topk_ids, topk_w, w13_blocks, w13_gscale, w2_blocks, w2_gscale, pw1, e_total):
    return x.new_empty(x.shape)


def forward(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, state: dict, e_total: int) -> torch.Tensor:
    return moe_w4a16(x, topk_ids.contiguous(), topk_w.contiguous(), state["w13_blocks"], state["w13_gscale"],
                     state["w2_blocks"], state["w2_gscale"], state["pw1"], int(e_total))
