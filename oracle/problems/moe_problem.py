"""Shared body of the kdev MoE problem references (decode / prefill / skewed configurations).
TEST INFRASTRUCTURE: imported only by oracle/problems/b200_moe_*/reference.py, the reference modules kdev's
OKC adapter loads (src/kdev/adapters/okc.py:476-575)."""
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parents[2]
for _p in (str(_ROOT), str(_ROOT / "kernel-development_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from kdb200 import workloads as W  # noqa: E402
from oracle import moe as om  # noqa: E402


def make(name: str) -> dict:
    cfg = W.MOE_CONFIGS[name]

    def _dev(device):
        return device if (device != "cuda" or torch.cuda.is_available()) else "cpu"

    def generate_weights(seed, device="cuda"):
        w = W.moe_weights(cfg, int(seed), _dev(device))
        w["top_k"] = cfg.k
        return w

    def generate_input(t, seed, device="cuda", **_):
        return {"x": W.moe_input(int(t), cfg.h, int(seed), _dev(device)), "config": {"t": int(t), "layer": name}}

    def check_implementation(data, output, weights):
        ref = om.moe_ref(data["x"], weights, cfg.k)
        return om.check(tuple(o.detach().cpu() for o in output), ref)

    def speed_of_light_ns(t, hw, **_):
        c = W.MoeConfig(name, int(t), cfg.h, cfg.e, cfg.i, cfg.k, cfg.shared, cfg.shared_i)
        distinct = min(cfg.e, int(t) * cfg.k)
        return 1e9 * max(W.moe_bytes(c, distinct) / hw["hbm_bytes_per_s"], W.moe_flops(c) / hw["bf16_dense_flops_per_s"])

    return {"WEIGHTS_SEED": 0, "TOP_K": cfg.k, "REL_L2_TOL": om.REL_FRO_TOL, "CONFIG": cfg,
            "generate_weights": generate_weights, "generate_input": generate_input,
            "check_implementation": check_implementation, "speed_of_light_ns": speed_of_light_ns}
