"""kdev problem reference for FP8-KV paged decode / verify attention.  TEST INFRASTRUCTURE: the checker kdev's
OKC adapter imports (src/kdev/adapters/okc.py:476-575, "attention: kernel_fn(data), no prepare/weights; check
via R.collect(data, out) then R.check_implementation(data, raw)"); the product never imports it.

Cases {"batch", "ctx", "heads", "layer", "q_len", "page", "spread", "dist", "kv_scale"} as in the reference's
problem (src/kdev/adapters/okc_problems/muse_attention_decode.toml); inputs and the check are the oracle's
(oracle/attention.py).  kernel_fn(data) appends the new tokens' K/V into data["k_cache"] / data["v_cache"] and
returns the output; collect() hands the check the output and both caches.
"""
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parents[3]
for _p in (str(_ROOT), str(_ROOT / "kernel-development_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from oracle import attention as oa  # noqa: E402

HEAD_DIM = oa.HEAD_DIM


def _dev(device):
    return device if (device != "cuda" or torch.cuda.is_available()) else "cpu"


def generate_input(batch, ctx, seed, heads="tp8", layer="full", q_len=1, page=1, spread="none", dist="soft",
                   kv_scale=1.0, device="cuda", **_):
    if int(page) != 1:
        raise ValueError("page size 1 only (the reference problem's cases)")
    case = oa.AttnCase(int(batch), int(ctx), heads, layer, int(q_len), 1, spread or "none", dist, float(kv_scale))
    data = oa.generate_input(case, int(seed))
    d = _dev(device)
    return {k: (v.to(d) if isinstance(v, torch.Tensor) else v) for k, v in data.items()}


def collect(data, out):
    if not isinstance(out, torch.Tensor) or tuple(out.shape) != tuple(data["q"].shape):
        raise ValueError(f"output must be a tensor of shape {tuple(data['q'].shape)}")
    return {"out": out, "k_cache": data["k_cache"], "v_cache": data["v_cache"]}


def check_implementation(data, got):
    cpu = {k: (v.detach().cpu() if isinstance(v, torch.Tensor) else v) for k, v in data.items()}
    kc, vc = oa.append_kv(cpu)
    for name, want in (("k_cache", kc), ("v_cache", vc)):
        if not torch.equal(got[name].detach().cpu().view(torch.uint8), want.view(torch.uint8)):
            return False, f"{name}: the new entries are not the FP8 E4M3 of value / kv_scale in their slots"
    return oa.check(cpu, got["out"].detach().cpu())
