# okc: problem=b200_attention_decode
"""kdev submission for FP8-KV paged decode / verify attention: `kernel_fn(data)` appends the new tokens' K/V
to data["k_cache"] / data["v_cache"] and returns out bf16 [batch, q_len, q_heads, 128].  The op is
kdb200.attention (libkdb200.so); there is no fallback path."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parent.parent)
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from kdb200 import attention as _attn  # noqa: E402


def kernel_fn(data):
    return _attn.decode(data["q"], data["k_new"], data["v_new"], data["k_cache"], data["v_cache"],
                        data["block_table"], data["seq_lens"], data["kv_scale"],
                        _attn.window_of(data["config"]["layer"]))
