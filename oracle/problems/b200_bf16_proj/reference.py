"""kdev problem reference for the B200 bf16 projection.  TEST INFRASTRUCTURE (the checker kdev's
OKC adapter imports: src/kdev/adapters/okc.py:476-575); the product never imports it.

API (the one kdev's OkcAdapter calls): generate_weights(seed), generate_input(m, layer, seed),
check_implementation(data, out, weights) -> (ok, msg), speed_of_light_ns(m, layer, hw).
Weights: one bf16 W[N, K] per layer; input {"x": bf16[m, K], "config": {"m", "layer"}}.
"""
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parents[3]
for _p in (str(_ROOT), str(_ROOT / "kernel-development_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from kdb200 import workloads as W  # noqa: E402
from oracle import proj as op  # noqa: E402

WEIGHTS_SEED = 0
REL_L2_TOL = op.REL_FRO_TOL
LAYERS = {"k2048_n2048": (2048, 2048), "k7168_n7168": (7168, 7168)}


def _dev(device):
    return device if (device != "cuda" or torch.cuda.is_available()) else "cpu"


def generate_weights(seed, device="cuda"):
    return {name: W.proj_weight(k, n, seed * 10 + i, _dev(device)) for i, (name, (k, n)) in enumerate(LAYERS.items())}


def generate_input(m, layer, seed, device="cuda", **_):
    k, _n = LAYERS[layer]
    return {"x": W.proj_input(int(m), k, int(seed), _dev(device)), "config": {"m": int(m), "layer": layer}}


def check_implementation(data, output, weights):
    w = weights[data["config"]["layer"]]
    if not isinstance(output, torch.Tensor):
        return False, "expected a tensor"
    return op.check(output.detach().cpu(), op.proj_ref(data["x"], w))


def speed_of_light_ns(m, layer, hw, **_):
    k, n = LAYERS[layer]
    cfg = W.ProjConfig("sol", int(m), k, n)
    return 1e9 * max(cfg.bytes() / hw["hbm_bytes_per_s"], cfg.flops() / hw["bf16_dense_flops_per_s"])
