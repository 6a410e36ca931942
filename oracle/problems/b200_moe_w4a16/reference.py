"""kdev problem reference for the NVFP4 w4a16 MoE layer of one ep8 rank.  TEST INFRASTRUCTURE: the
checker kdev's OKC adapter imports (src/kdev/adapters/okc.py:476-575); the product never imports it.

Cases {"bs": tokens, "sharding": "ep8"[, "dist": "skewed"]}, as in the reference's problem list
(src/kdev/adapters/okc_problems/muse_moe_w4a16.toml).  Weights: NVFP4 local experts (kdb200.workloads.
w4a16_weights); input: x bf16 [bs, H] and routing over all experts with this rank the busiest.
"""
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parents[3]
for _p in (str(_ROOT), str(_ROOT / "kernel-development_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from kdb200 import workloads as W  # noqa: E402
from oracle import moe_w4a16 as ow  # noqa: E402

WEIGHTS_SEED = 0
CONFIG = W.W4A16_CONFIGS["w4a16_bs16"]
REL_L2_TOL = ow.REL_FRO_TOL


def _dev(device):
    return device if (device != "cuda" or torch.cuda.is_available()) else "cpu"


def generate_weights(seed, device="cuda"):
    w = W.w4a16_weights(CONFIG, int(seed))
    w = {k: v.to(_dev(device)) for k, v in w.items()}
    w["e_total"] = CONFIG.e_total
    return w


def generate_input(bs, seed, sharding="ep8", device="cuda", dist="normal", **_):
    cfg = W.W4A16Config("case", int(bs), CONFIG.h, CONFIG.i, CONFIG.local, CONFIG.e_total, CONFIG.k,
                        skew=(dist == "skewed"))
    ids, tw = W.w4a16_routing(cfg, int(seed))
    d = _dev(device)
    return {"x": W.moe_input(int(bs), CONFIG.h, int(seed), d), "topk_ids": ids.to(d), "topk_w": tw.to(d),
            "config": {"bs": int(bs), "sharding": sharding, "dist": dist}}


def check_implementation(data, output, weights):
    cpu = {k: (v.detach().cpu() if isinstance(v, torch.Tensor) else v) for k, v in weights.items()}
    ref = ow.w4a16_ref(data["x"], data["topk_ids"], data["topk_w"], cpu, CONFIG.local)
    return ow.check(output, ref)


def speed_of_light_ns(bs, hw, **_):
    # the NVFP4 bytes of the local experts a batch of bs tokens can reach (at most all of them)
    per_expert = 3 * CONFIG.h * CONFIG.i * (0.5 + 1 / 16)
    hit = min(CONFIG.local, int(bs) * CONFIG.k)
    return 1e9 * hit * per_expert / hw["hbm_bytes_per_s"]
