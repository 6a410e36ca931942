"""bf16 dense projection Y = X · Wᵀ as a PyTorch custom op over libkdb200.

Forward signature follows the reference's `muse_bf16_proj` problem: kdev calls
`kernel_fn(data, state)` with data = {"x": bf16[M, K], "config": {...}} and state = prepare(weights)
(src/kdev/adapters/okc.py:501-537).  `proj(x, w)` is the op behind that kernel_fn.
"""
from __future__ import annotations

import torch

from . import _lib


def _check_operand(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be row-major contiguous")


def proj_into(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, tile_n: int = 0, cta_pair: int = 0) -> torch.Tensor:
    """Writes X · Wᵀ into `y` ([M, N] bf16; a column slice of a wider row-major matrix is allowed).
    tile_n / cta_pair force the tile shape (0 = automatic; cta_pair=1: 256-row tiles on CTA pairs)."""
    _check_operand("x", x)
    _check_operand("w", w)
    m, k = x.shape
    n, k2 = w.shape
    if k != k2:
        raise ValueError(f"x is [{m}, {k}] but w is [{n}, {k2}]: K mismatch")
    if y.dtype != torch.bfloat16 or y.dim() != 2 or tuple(y.shape) != (m, n) or y.stride(1) != 1:
        raise ValueError(f"y must be bf16 [{m}, {n}] with unit column stride")
    if not (x.device == w.device == y.device):
        raise ValueError("x, w and y must be on the same device")
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        if tile_n == 0 and cta_pair == 0:
            # automatic shape; small-M shapes split K and sum fp32 partials from a workspace
            nbytes = int(_lib.lib().kdb_proj_workspace_bytes(m, n, k)) if m > 0 and n > 0 and k > 0 else 0
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device) if nbytes else None
            rc = _lib.lib().kdb_proj_bf16_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, y.stride(0),
                                             None if ws is None else ws.data_ptr(), nbytes, stream)
        else:
            rc = _lib.lib().kdb_proj_bf16_cfg(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, y.stride(0),
                                              int(tile_n), int(cta_pair), stream)
    _lib.check("kdb_proj_bf16", rc)
    return y


def tile_shape(m: int, n: int) -> tuple[int, bool]:
    """(tile width, CTA pair) the projection picks for an m x n output on the current device."""
    import ctypes
    out = (ctypes.c_int32 * 2)()
    _lib.check("kdb_proj_tile_shape", _lib.lib().kdb_proj_tile_shape(m, n, out))
    return int(out[0]), bool(out[1])


@torch.library.custom_op("kdb200::proj", mutates_args=())
def proj(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Y[M, N] = X[M, K] · W[N, K]ᵀ, bf16 in/out, fp32 accumulation (tcgen05 on sm_100a)."""
    y = torch.empty((x.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    return proj_into(x, w, y)


@proj.register_fake
def _proj_fake(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return x.new_empty((x.shape[0], w.shape[0]))


# ------------------------------------------------------------------------- fp32 weights (router layer)
def split_f32(w: torch.Tensor) -> torch.Tensor:
    """w fp32 [N, K] -> w_split bf16 [N, 2K] = [bf16(W) | bf16(W - bf16(W))] per row (prepare step of the
    router layer: "fp32 weights and output (BF16 hi+lo pair with FP32 accumulation allowed)",
    src/kdev/adapters/okc_problems/muse_bf16_proj.toml:371).  The caller's w is not modified."""
    if not w.is_cuda or w.dtype != torch.float32 or w.dim() != 2:
        raise TypeError("w must be a 2-D fp32 CUDA tensor")
    w = w.contiguous()
    n, k = w.shape
    out = torch.empty((n, 2 * k), dtype=torch.bfloat16, device=w.device)
    with torch.cuda.device(w.device):
        rc = _lib.lib().kdb_proj_split_f32(w.data_ptr(), out.data_ptr(), n, k,
                                           torch.cuda.current_stream(w.device).cuda_stream)
    _lib.check("kdb_proj_split_f32", rc)
    return out


@torch.library.custom_op("kdb200::proj_f32w", mutates_args=())
def proj_f32w(x: torch.Tensor, w_split: torch.Tensor) -> torch.Tensor:
    """Y fp32 [M, N] = X[M, K] · (W_hi + W_mid)ᵀ, w_split = split_f32(W) ([N, 2K] bf16), fp32 accumulation."""
    _check_operand("x", x)
    _check_operand("w_split", w_split)
    m, k = x.shape
    n, k2 = w_split.shape
    if k2 != 2 * k:
        raise ValueError(f"x is [{m}, {k}] but w_split is [{n}, {k2}]: expected [{n}, {2 * k}]")
    if w_split.device != x.device:
        raise ValueError("x and w_split must be on the same device")
    y = torch.empty((m, n), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        nbytes = int(_lib.lib().kdb_proj_f32w_workspace_bytes(m, n, k)) if m > 0 and n > 0 and k > 0 else 0
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device) if nbytes else None
        rc = _lib.lib().kdb_proj_f32w(x.data_ptr(), w_split.data_ptr(), y.data_ptr(), m, n, k,
                                      None if ws is None else ws.data_ptr(), nbytes,
                                      torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check("kdb_proj_f32w", rc)
    return y


@proj_f32w.register_fake
def _proj_f32w_fake(x: torch.Tensor, w_split: torch.Tensor) -> torch.Tensor:
    return x.new_empty((x.shape[0], w_split.shape[0]), dtype=torch.float32)
