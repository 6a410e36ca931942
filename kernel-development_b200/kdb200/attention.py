"""Paged decode / verify attention over an FP8 E4M3 KV cache as a PyTorch custom op over libkdb200
(kdb_attn_decode_fp8): the reference's `muse_attention_decode` problem
(src/kdev/adapters/okc_problems/muse_attention_decode.toml), where kernel_fn(data) appends the new tokens'
K/V to the cache and returns the attention output.

decode(q, k_new, v_new, k_cache, v_cache, block_table, seq_lens, kv_scale, window) writes the new entries
into k_cache / v_cache (in place) and returns out bf16 [B, q_len, Hq, 128].  window = 2048 for a sliding
layer, 0 for a full one.
"""
from __future__ import annotations

import torch

from . import _lib

HEAD_DIM = 128
SLIDING_WINDOW = 2048


def _check(q, k_new, v_new, k_cache, v_cache, block_table, seq_lens):
    """Shapes, dtypes and devices; returns (B, T, Hq, Hkv, max_len, slots).  The kernels receive raw pointers,
    so every tensor must be contiguous and on q's CUDA device."""
    if q.dtype != torch.bfloat16 or q.dim() != 4 or q.shape[-1] != HEAD_DIM:
        raise TypeError(f"q must be bf16 [B, q_len, q_heads, {HEAD_DIM}]")
    if k_new.dtype != torch.bfloat16 or v_new.dtype != torch.bfloat16 or k_new.shape != v_new.shape:
        raise TypeError("k_new and v_new must be bf16 [B, q_len, kv_heads, 128] of one shape")
    if k_cache.dtype != torch.float8_e4m3fn or v_cache.dtype != torch.float8_e4m3fn or k_cache.shape != v_cache.shape:
        raise TypeError("k_cache and v_cache must be float8_e4m3fn [slots, kv_heads, 128] of one shape")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_table and seq_lens must be int32")
    B, T, Hq, D = q.shape
    slots, Hkv, _ = k_cache.shape
    if tuple(k_new.shape) != (B, T, Hkv, D) or k_cache.shape[-1] != D:
        raise ValueError(f"k_new {tuple(k_new.shape)} / k_cache {tuple(k_cache.shape)} do not match q {tuple(q.shape)}")
    if block_table.dim() != 2 or block_table.shape[0] != B or tuple(seq_lens.shape) != (B,):
        raise ValueError("block_table must be [B, max_len] and seq_lens [B]")
    if Hq % Hkv:
        raise ValueError(f"q_heads ({Hq}) must be a multiple of kv_heads ({Hkv})")
    tensors = (q, k_new, v_new, k_cache, v_cache, block_table, seq_lens)
    if not q.is_cuda or any(a.device != q.device for a in tensors):
        raise ValueError("all tensors must be on one CUDA device (there is no CPU path)")
    if not all(a.is_contiguous() for a in tensors):
        raise ValueError("all tensors must be contiguous")
    return B, T, Hq, Hkv, block_table.shape[1], slots


@torch.library.custom_op("kdb200::attn_decode_fp8", mutates_args=("k_cache", "v_cache"))
def attn_decode_fp8(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor, kv_scale: float,
                    window: int) -> torch.Tensor:
    """out bf16 [B, q_len, Hq, 128]; appends k_new / v_new (e4m3 of value / kv_scale) into the caches first."""
    B, T, Hq, Hkv, max_len, slots = _check(q, k_new, v_new, k_cache, v_cache, block_table, seq_lens)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    nbytes = int(_lib.lib().kdb_attn_decode_workspace_bytes(B, T, Hq, Hkv, max_len, window))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = _lib.lib().kdb_attn_decode_fp8(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            block_table.data_ptr(), seq_lens.data_ptr(), float(kv_scale), out.data_ptr(), B, T, Hq, Hkv, HEAD_DIM,
            max_len, slots, int(window), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check("kdb_attn_decode_fp8", rc)
    return out


@attn_decode_fp8.register_fake
def _attn_decode_fp8_fake(q, k_new, v_new, k_cache, v_cache, block_table, seq_lens, kv_scale, window):
    return q.new_empty(q.shape)


def decode(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
           block_table: torch.Tensor, seq_lens: torch.Tensor, kv_scale: float = 1.0, window: int = 0) -> torch.Tensor:
    return attn_decode_fp8(q.contiguous(), k_new.contiguous(), v_new.contiguous(), k_cache, v_cache,
                           block_table.contiguous(), seq_lens.contiguous(), float(kv_scale), int(window))


def window_of(layer: str) -> int:
    """The key window of a layer kind: 2048 for "sliding", 0 (the whole context) for "full"."""
    if layer not in ("sliding", "full"):
        raise ValueError(f"unknown layer {layer!r}")
    return SLIDING_WINDOW if layer == "sliding" else 0
