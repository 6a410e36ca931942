"""oracle — CPU restatement of the two hot paths.  TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package, and only
to verify GPU results (or as the timed CPU baseline).  The product path (kernel-development_b200/kdb200 and
libkdb200.so) never imports, links or executes anything here.

What it restates:
  proj.py     Y = X · Wᵀ in fp32 from bf16 operands (the `muse_bf16_proj` problem's math,
              src/kdev/adapters/okc_problems/muse_bf16_proj.toml:1-8; fp32 accumulate, bf16 out).
  moe.py      the MoE layer: fp32 router -> softmax -> top-k -> renormalised weights; grouped
              SwiGLU experts (gate_up, silu(g)*u rounded to bf16, down); weighted combine; shared
              expert.  Structure follows the reference engine's plan/expert/combine stages
              (okc-challenge/engines/x3_h.cu:346-385 plan, sc_h.cu:322-340 SwiGLU epilogue,
              sc_h.cu:374-381 weighted combine), with the math of the bf16 layer.
  routing.c   the integer/bit-exact part of routing in C: fixed-order fp64 router logits, top-k,
              the stable (expert, token) permutation.  Built by oracle/build.py.
  moe_w4a16.py  the NVFP4 w4a16 MoE layer of one expert-parallel rank (post-expert RMS norm).
  attention.py  fp8-KV paged decode / verify attention with its check (no GPU kernel for it yet).
  problems/   kdev problem dirs (TASK.md + reference.py) and TOMLs so kdev's OKC adapter, `kdev check`
              and `kdev ab` drive the ops unchanged.

PARITY UNPINNED.  The reference ships no golden vectors, known-answer tests or fixtures for these
paths: the OKC problems' own reference.py/checks.py are not in the reference tree
(src/kdev/adapters/okc.py:3-5, 71-87), and its only kernels (okc-challenge/engines/*.cu) are
GPU-only NVFP4 engines with different math.  The golden files under tests/golden/ are generated from
this oracle (tests/golden/make_golden.py) and pin it against drift, not against the reference.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent

_routing = None


def routing_lib() -> ctypes.CDLL:
    """The compiled routing.c (built on first use)."""
    global _routing
    if _routing is None:
        from .build import build
        lib = ctypes.CDLL(str(build()))
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.oracle_router_logits.argtypes = [vp, vp, vp, i64, i64, i64, vp]
        lib.oracle_router_logits.restype = None
        lib.oracle_topk.argtypes = [vp, i64, i64, i32, vp, vp]
        lib.oracle_topk.restype = None
        lib.oracle_permute.argtypes = [vp, i64, i32, i64, vp, vp, vp, vp]
        lib.oracle_permute.restype = i32
        _routing = lib
    return _routing
