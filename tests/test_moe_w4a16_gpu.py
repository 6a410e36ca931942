"""GPU parity tests of the NVFP4 w4a16 MoE layer (kdb_moe_w4a16_forward) against the fp32 oracle
(oracle/moe_w4a16.py).  Tolerance (written here, the oracle's): max-abs <= 2e-2 and relative Frobenius
<= 1e-2 of the output."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest
import torch

from kdb200 import moe_w4a16 as W4
from kdb200 import workloads as W
from oracle import moe_w4a16 as ow

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _run(cfg, seed=1, x=None, ids=None, tw=None):
    wts = W.w4a16_weights(cfg, seed)
    if ids is None:
        ids, tw = W.w4a16_routing(cfg, seed)
    if x is None:
        x = W.moe_input(cfg.t, cfg.h, seed)
    state = W4.prepare(wts)
    y = W4.forward(x.cuda(), ids.cuda(), tw.cuda(), state, cfg.e_total)
    torch.cuda.synchronize()
    return y, ow.w4a16_ref(x, ids, tw, wts, cfg.local), (x, ids, tw, wts, state)


@pytest.mark.parametrize("cfg", [
    W.W4A16Config("tiny", 8, 256, 128, 4, 32, 4),
    W.W4A16Config("skew", 33, 512, 256, 8, 64, 8, skew=True),
    W.W4A16Config("many_per_expert", 150, 256, 128, 2, 8, 4),     # > 64 tokens of one expert: several token tiles
    W.W4A16Config("h4096", 16, 4096, 512, 8, 64, 8),
])
def test_w4a16_matches_oracle(cfg):
    y, ref, _ = _run(cfg)
    ok, msg = ow.check(y, ref)
    assert ok, msg


def test_w4a16_full_size_bs1():
    """H = I = 4096, 32 local of 256 experts, one token."""
    cfg = W.W4A16_CONFIGS["w4a16_bs1"]
    y, ref, _ = _run(cfg, seed=3)
    ok, msg = ow.check(y, ref)
    assert ok, msg


def test_w4a16_no_local_routes_gives_zeros_and_empty_batch():
    cfg = W.W4A16Config("none", 5, 256, 128, 4, 32, 4)
    ids = torch.arange(4, 24, dtype=torch.int32).view(5, 4)          # every route goes to another rank
    tw = torch.full((5, 4), 0.25)
    y, ref, _ = _run(cfg, ids=ids, tw=tw)
    assert torch.equal(y.cpu(), torch.zeros_like(y.cpu())) and float(ref.abs().max()) == 0.0
    cfg0 = W.W4A16Config("empty", 0, 256, 128, 4, 32, 4)
    state = W4.prepare(W.w4a16_weights(cfg0, 1))
    y0 = W4.forward(torch.empty((0, 256), dtype=torch.bfloat16, device="cuda"),
                    torch.empty((0, 4), dtype=torch.int32, device="cuda"),
                    torch.empty((0, 4), dtype=torch.float32, device="cuda"), state, 32)
    assert y0.shape == (0, 256)


def test_w4a16_graph_replay_and_determinism():
    cfg = W.W4A16Config("graph", 40, 512, 256, 8, 64, 8)
    y, ref, (x, ids, tw, _, state) = _run(cfg, seed=5)
    gx, gi, gw = x.cuda(), ids.cuda(), tw.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        W4.forward(gx, gi, gw, state, cfg.e_total)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = W4.forward(gx, gi, gw, state, cfg.e_total)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y)
    y2 = W4.forward(gx, gi, gw, state, cfg.e_total)
    torch.cuda.synchronize()
    assert torch.equal(y2, y)


def test_w4a16_through_submission():
    spec = importlib.util.spec_from_file_location(
        "b200_moe_w4a16_sub", ROOT / "kernel-development_b200" / "submissions" / "b200_moe_w4a16.py")
    sub = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sub)
    cfg = W.W4A16Config("sub", 12, 512, 256, 8, 64, 8)
    wts = W.w4a16_weights(cfg, 2)
    wts_dev = {k: v.cuda() for k, v in wts.items()}
    wts_dev["e_total"] = cfg.e_total
    before = {k: v.clone() for k, v in wts_dev.items() if isinstance(v, torch.Tensor)}
    state = sub.prepare(wts_dev)
    for k, v in before.items():
        assert torch.equal(v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v,
                           wts_dev[k].view(torch.uint8) if v.dtype == torch.float8_e4m3fn else wts_dev[k])
    ids, tw = W.w4a16_routing(cfg, 2)
    x = W.moe_input(cfg.t, cfg.h, 2)
    y = sub.kernel_fn({"x": x.cuda(), "topk_ids": ids.cuda(), "topk_w": tw.cuda(), "config": {"bs": cfg.t}}, state)
    torch.cuda.synchronize()
    ok, msg = ow.check(y, ow.w4a16_ref(x, ids, tw, wts, cfg.local))
    assert ok, msg


def test_w4a16_per_feature_weight_pw1():
    """The engines' per-feature output weight pw1 (okc-challenge/engines/sc_h.cu:51, 346) multiplies y before
    its sum of squares: with a non-unit pw1 the output matches the oracle and differs from pw1 = 1."""
    cfg = W.W4A16Config("pw1", 24, 512, 256, 4, 32, 4)
    wts = W.w4a16_weights(cfg, 5)
    assert float((wts["pw1"] - 1).abs().max()) > 0.1
    ids, tw = W.w4a16_routing(cfg, 5)
    x = W.moe_input(cfg.t, cfg.h, 5)
    y = W4.forward(x.cuda(), ids.cuda(), tw.cuda(), W4.prepare(wts), cfg.e_total)
    ones = dict(wts, pw1=torch.ones(cfg.h))
    y1 = W4.forward(x.cuda(), ids.cuda(), tw.cuda(), W4.prepare(ones), cfg.e_total)
    torch.cuda.synchronize()
    ok, msg = ow.check(y, ow.w4a16_ref(x, ids, tw, wts, cfg.local))
    assert ok, msg
    ok1, msg1 = ow.check(y1, ow.w4a16_ref(x, ids, tw, ones, cfg.local))
    assert ok1, msg1
    assert float((y.float() - y1.float()).abs().max()) > 0.05
