"""kdev problem reference for the B200 bf16 projection.  TEST INFRASTRUCTURE (the reference module kdev's
OKC adapter imports: src/kdev/adapters/okc.py:476-575); the product never imports it.

API (the one kdev's OkcAdapter calls): generate_weights(seed), generate_input(m, layer, seed),
check_implementation(data, out, weights) -> (ok, msg), speed_of_light_ns(m, layer, hw).
Weights: one bf16 W[N, K] per layer, and fp32 W for the "router" layer (the reference's precision rule:
fp32 weights and output, BF16 hi+lo pair with FP32 accumulation allowed, muse_bf16_proj.toml:371);
input {"x": bf16[m, K], "config": {"m", "layer"[, "dist"]}}.
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
LAYERS = {"k2048_n2048": (2048, 2048), "k7168_n7168": (7168, 7168), "router": (7168, 256)}
FP32_LAYERS = {"router"}


def _dev(device):
    return device if (device != "cuda" or torch.cuda.is_available()) else "cpu"


def generate_weights(seed, device="cuda"):
    out = {}
    for i, (name, (k, n)) in enumerate(LAYERS.items()):
        gen = W.proj_weight_f32 if name in FP32_LAYERS else W.proj_weight
        out[name] = gen(k, n, seed * 10 + i, _dev(device))
    return out


def generate_input(m, layer, seed, device="cuda", dist="normal", **_):
    k, _n = LAYERS[layer]
    cfg = {"m": int(m), "layer": layer}
    if dist != "normal":
        cfg["dist"] = dist
    return {"x": W.proj_input(int(m), k, int(seed), _dev(device), dist), "config": cfg}


def check_implementation(data, output, weights):
    layer = data["config"]["layer"]
    w = weights[layer]
    if not isinstance(output, torch.Tensor):
        return False, "expected a tensor"
    if layer in FP32_LAYERS:
        return op.check_f32w(output.detach().cpu(), op.proj_ref_f32w(data["x"], w))
    return op.check(output.detach().cpu(), op.proj_ref(data["x"], w))


def speed_of_light_ns(m, layer, hw, **_):
    k, n = LAYERS[layer]
    cfg = W.ProjConfig("sol", int(m), k, n)
    return 1e9 * max(cfg.bytes() / hw["hbm_bytes_per_s"], cfg.flops() / hw["bf16_dense_flops_per_s"])
