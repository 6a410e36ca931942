# okc: problem=b200_moe_skewed
"""kdev submission for the fused MoE layer (skewed configuration): `prepare(weights)` packs the
gate/up rows once (untimed), `kernel_fn(data, state)` returns (y, topk_w, topk_ids) with the routing
ids at output index 2.  The op is kdb200.moe (libkdb200.so); there is no fallback path."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parent.parent)
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from kdb200 import moe as _moe  # noqa: E402


def prepare(weights):
    return _moe.prepare(weights, int(weights["top_k"]))


def kernel_fn(data, state):
    return _moe.forward(data["x"], state)
