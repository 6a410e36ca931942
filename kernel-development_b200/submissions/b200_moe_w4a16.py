# okc: problem=b200_moe_w4a16
"""kdev submission for the NVFP4 w4a16 MoE layer of one ep8 rank: `prepare(weights)` tiles the NVFP4
weights losslessly (untimed), `kernel_fn(data, state)` returns y bf16 [bs, H].  The op is
kdb200.moe_w4a16 (libkdb200.so); there is no fallback path."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parent.parent)
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from kdb200 import moe_w4a16 as _w4  # noqa: E402


def prepare(weights):
    state = _w4.prepare(weights)
    state["e_total"] = int(weights["e_total"])
    return state


def kernel_fn(data, state):
    return _w4.forward(data["x"], data["topk_ids"], data["topk_w"], state, state["e_total"])
