"""Generate the golden fixtures in this directory from the oracle (fixed seeds).

    python tests/golden/make_golden.py

The reference ships no golden vectors for these paths (its OKC problem references are not in its
tree), so these fixtures pin the oracle against drift and give the GPU tests stored expected
outputs; they do not pin parity with the reference.  Each .npz holds the inputs (bf16 stored as
uint16 bits) and the oracle's outputs; manifest.json holds their sha256.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (str(ROOT), str(ROOT / "kernel-development_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from kdb200 import workloads as W  # noqa: E402
from oracle import moe as om  # noqa: E402
from oracle import proj as op  # noqa: E402

ROUTING_CASES = [
    {"name": "route_small", "t": 64, "h": 256, "e": 16, "k": 4, "seed": 11, "zipf": 0.0, "ties": False},
    {"name": "route_skew", "t": 256, "h": 512, "e": 64, "k": 4, "seed": 12, "zipf": 1.2, "ties": False},
    {"name": "route_ties", "t": 32, "h": 64, "e": 8, "k": 3, "seed": 13, "zipf": 0.0, "ties": True},
    {"name": "route_odd", "t": 7, "h": 40, "e": 5, "k": 5, "seed": 14, "zipf": 0.0, "ties": False},
]
LAYER_CASES = [
    {"name": "layer_small", "t": 24, "h": 128, "e": 8, "i": 128, "k": 2, "shared": 0, "shared_i": 0, "seed": 21},
    {"name": "layer_shared", "t": 16, "h": 256, "e": 4, "i": 128, "k": 2, "shared": 1, "shared_i": 128, "seed": 22},
]
PROJ_CASES = [
    {"name": "proj_small", "m": 32, "k": 64, "n": 48, "seed": 31},
    {"name": "proj_ragged", "m": 37, "k": 136, "n": 72, "seed": 32},
]


def routing_inputs(case):
    cfg = W.MoeConfig(case["name"], case["t"], case["h"], case["e"], 128, case["k"], zipf_s=case["zipf"])
    x = W.moe_input(cfg.t, cfg.h, case["seed"])
    router = W._randn((cfg.e, cfg.h), case["seed"] * 1000 + 3, "cpu", 1.0 / cfg.h ** 0.5, torch.float32)
    if case["ties"]:
        router[5] = router[3]          # identical rows: equal logits, lower expert must win
        router[7] = router[3]
    bias = W.zipf_router_bias(cfg.e, cfg.zipf_s, case["seed"]) if cfg.zipf_s > 0 else None
    return x, {"router": router, "router_bias": bias}


def layer_inputs(case):
    cfg = W.MoeConfig(case["name"], case["t"], case["h"], case["e"], case["i"], case["k"], case["shared"],
                      case["shared_i"])
    return W.moe_input(cfg.t, cfg.h, case["seed"]), W.moe_weights(cfg, case["seed"]), cfg


def proj_inputs(case):
    return W.proj_input(case["m"], case["k"], case["seed"]), W.proj_weight(case["k"], case["n"], case["seed"])


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    files = {}
    for case in ROUTING_CASES:
        x, wts = routing_inputs(case)
        lg = om.router_logits(x, wts["router"], wts["router_bias"])
        ids, _ = om.topk(lg, case["k"])
        w = om.renorm_weights(lg, ids)
        p = om.permute(ids, case["e"])
        arrs = {"x_bits": _bits(x), "router": wts["router"].numpy(), "logits": lg.numpy(), "ids": ids.numpy(),
                "w": w.numpy(), "perm_slot": p["perm_slot"].numpy(), "slot_pos": p["slot_pos"].numpy(),
                "counts": p["counts"].numpy(), "offsets": p["offsets"].numpy()}
        if wts["router_bias"] is not None:
            arrs["router_bias"] = wts["router_bias"].numpy()
        files[case["name"]] = arrs
    for case in LAYER_CASES:
        x, wts, cfg = layer_inputs(case)
        ref = om.moe_ref(x, wts, cfg.k)
        arrs = {"x_bits": _bits(x), "router": wts["router"].numpy(), "w_gate_up_bits": _bits(wts["w_gate_up"]),
                "w_down_bits": _bits(wts["w_down"]), "ids": ref["ids"].numpy(), "w": ref["w"].numpy(),
                "y32": ref["y32"].numpy(), "y_bits": _bits(ref["y"])}
        if wts["shared_gate_up"] is not None:
            arrs["shared_gate_up_bits"] = _bits(wts["shared_gate_up"])
            arrs["shared_down_bits"] = _bits(wts["shared_down"])
        files[case["name"]] = arrs
    for case in PROJ_CASES:
        x, w = proj_inputs(case)
        files[case["name"]] = {"x_bits": _bits(x), "w_bits": _bits(w), "y32": op.proj_ref(x, w).numpy()}
    manifest = {"generator": "tests/golden/make_golden.py", "files": {}}
    for name, arrs in files.items():
        path = HERE / f"{name}.npz"
        np.savez(path, **arrs)
        manifest["files"][path.name] = hashlib.sha256(path.read_bytes()).hexdigest()
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(files)} fixtures")


if __name__ == "__main__":
    main()
