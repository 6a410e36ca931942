"""kdb200 — B200 (sm_100a) bf16 projection and fused MoE layer behind kdev's problem-adapter API.

Host-side layer over libkdb200.so (include/kdb200.h).  Public surface:
  proj(x, w), proj_into(x, w, y)             bf16 dense projection (torch op kdb200::proj)
  moe.*                                       fused MoE layer (router, permute, grouped GEMMs, combine)
  submissions/*.py                            kdev submission files: prepare(weights), kernel_fn(data, state)
"""
from . import _lib
from .proj import proj, proj_f32w, proj_into, split_f32

__all__ = ["proj", "proj_into", "proj_f32w", "split_f32", "_lib"]
