# okc: problem=b200_bf16_proj
"""kdev submission for the bf16 projection: `prepare(weights)` and `kernel_fn(data, state)`, the two
names kdev's OKC adapter calls (src/kdev/adapters/okc.py:501-537).  The op is kdb200.proj, a
tcgen05 GEMM in libkdb200.so; there is no fallback path."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parent.parent)
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from kdb200 import proj as _proj  # noqa: E402


def prepare(weights):
    """Weights are kept as given (bf16, bit-exact); one contiguous [N, K] tensor per layer."""
    return {layer: w.contiguous() for layer, w in weights.items()}


def kernel_fn(data, state):
    return _proj(data["x"], state[data["config"]["layer"]])
