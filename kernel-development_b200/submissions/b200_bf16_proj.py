# okc: problem=b200_bf16_proj
"""kdev submission for the bf16 projection: `prepare(weights)` and `kernel_fn(data, state)`, the two
names kdev's OKC adapter calls (src/kdev/adapters/okc.py:501-537).  The op is kdb200.proj, a
tcgen05 GEMM in libkdb200.so; there is no fallback path."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parent.parent)
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import torch  # noqa: E402

from kdb200 import proj as _proj  # noqa: E402
from kdb200 import proj_f32w as _proj_f32w  # noqa: E402
from kdb200 import split_f32 as _split_f32  # noqa: E402


def prepare(weights):
    """bf16 layers are kept as given (bit-exact, one contiguous [N, K] tensor each); an fp32 layer (the
    router) is stored as its lossless-to-2^-16 bf16 hi+mid pair [N, 2K] next to the untouched original."""
    state = {}
    for layer, w in weights.items():
        if w.dtype == torch.float32:
            state[layer] = ("f32", _split_f32(w))
        else:
            state[layer] = ("bf16", w.contiguous())
    return state


def kernel_fn(data, state):
    kind, w = state[data["config"]["layer"]]
    if kind == "f32":
        return _proj_f32w(data["x"], w)
    return _proj(data["x"], w)
