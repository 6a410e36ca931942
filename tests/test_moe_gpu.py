"""GPU parity tests of the MoE layer (libkdb200 kdb_moe_route / kdb_moe_plan / kdb_moe_forward)
against the oracle.

Bars: router logits bit-exact (fixed fp64 order), top-k ids and the permutation plan exact,
routing weights within 1e-6 absolute, layer output within max-abs 2e-2 AND relative Frobenius 1e-2
of the fp32 oracle."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from kdb200 import moe as M
from kdb200 import workloads as W
from oracle import moe as om

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
MAX_ABS = 2e-2
REL_FRO = 1e-2
W_ATOL = 1e-6


def _to_dev(wts):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in wts.items()}


def _route_and_plan_exact(x, wts, k, e):
    gx, gw = x.cuda(), _to_dev(wts)
    lg, w, ids = M.route(gx, gw["router"], gw.get("router_bias"), k)
    olg, oids, ow = om.route(x, wts["router"], wts.get("router_bias"), k)
    assert torch.equal(lg.cpu().view(torch.int32), olg.view(torch.int32)), "router logits not bit-exact"
    assert torch.equal(ids.cpu(), oids), "top-k ids differ"
    assert float((w.cpu() - ow).abs().max()) <= W_ATOL
    p = M.plan(ids, w, e)
    op_ = om.permute(oids, e)
    for name in ("counts", "offsets", "perm_slot", "slot_pos"):
        assert torch.equal(p[name].cpu(), op_[name]), name
    return olg, oids, ow


def _layer(cfg, seed):
    x = W.moe_input(cfg.t, cfg.h, seed)
    wts = W.moe_weights(cfg, seed)
    return x, wts


def _check_layer(x, wts, cfg):
    route = _route_and_plan_exact(x, wts, cfg.k, cfg.e)
    state = M.prepare(_to_dev(wts), cfg.k)
    y, w, ids = M.forward(x.cuda(), state)
    torch.cuda.synchronize()
    ref = om.moe_ref(x, wts, cfg.k, route_out=route)
    assert torch.equal(ids.cpu(), ref["ids"])
    c = om.compare(y, ref["y32"])
    assert c["nonfinite"] == 0 and c["max_abs"] <= MAX_ABS and c["rel_fro"] <= REL_FRO, c
    ok, msg = om.check((y, w, ids), ref)
    assert ok, msg
    return y, w, ids


@pytest.mark.parametrize("cfg", [
    W.MoeConfig("small", 100, 512, 16, 256, 4),
    W.MoeConfig("shared", 77, 256, 8, 128, 2, shared=1, shared_i=256),
    W.MoeConfig("k1", 50, 128, 4, 128, 1),
    W.MoeConfig("k_eq_e", 33, 128, 6, 128, 6),
    W.MoeConfig("one_token", 1, 256, 8, 128, 2),
    W.MoeConfig("odd_e", 300, 520, 37, 384, 8),         # E not a multiple of 16, H not of 256
    W.MoeConfig("many_tokens", 1500, 256, 64, 128, 8),  # several plan chunks
    W.MoeConfig("skew", 2048, 512, 128, 256, 4, zipf_s=1.2),
])
def test_layer_matches_oracle(cfg):
    x, wts = _layer(cfg, seed=cfg.t + cfg.e)
    _check_layer(x, wts, cfg)


def test_decode_config():
    """The decode configuration itself: T=64, H=4096, E=64, I=1024, top-8."""
    cfg = W.MOE_CONFIGS["moe_decode"]
    x, wts = _layer(cfg, seed=1)
    _check_layer(x, wts, cfg)


def test_routing_ties_lower_expert_wins():
    f = np.load(GOLDEN / "route_ties.npz")
    x = torch.from_numpy(f["x_bits"].view(np.int16)).view(torch.bfloat16)
    router = torch.from_numpy(f["router"])
    lg, w, ids = M.route(x.cuda(), router.cuda(), None, 3)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), f["ids"])
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), f["logits"].view(np.uint32))


@pytest.mark.parametrize("name", ["route_small", "route_skew", "route_odd"])
def test_golden_routing(name):
    f = np.load(GOLDEN / f"{name}.npz")
    x = torch.from_numpy(f["x_bits"].view(np.int16)).view(torch.bfloat16).cuda()
    router = torch.from_numpy(f["router"]).cuda()
    bias = torch.from_numpy(f["router_bias"]).cuda() if "router_bias" in f.files else None
    k = f["ids"].shape[1]
    e = f["counts"].shape[0]
    lg, w, ids = M.route(x, router, bias, k)
    p = M.plan(ids, w, e)
    torch.cuda.synchronize()
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), f["logits"].view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), f["ids"])
    assert np.array_equal(p["perm_slot"].cpu().numpy(), f["perm_slot"])
    assert np.array_equal(p["offsets"].cpu().numpy(), f["offsets"])
    assert np.allclose(w.cpu().numpy(), f["w"], atol=W_ATOL)


@pytest.mark.parametrize("name", ["layer_small", "layer_shared"])
def test_golden_layer(name):
    f = np.load(GOLDEN / f"{name}.npz")
    bf = lambda a: torch.from_numpy(f[a].view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    wts = {"router": torch.from_numpy(f["router"]).cuda(), "router_bias": None,
           "w_gate_up": bf("w_gate_up_bits"), "w_down": bf("w_down_bits"),
           "shared_gate_up": bf("shared_gate_up_bits") if "shared_gate_up_bits" in f.files else None,
           "shared_down": bf("shared_down_bits") if "shared_down_bits" in f.files else None}
    k = f["ids"].shape[1]
    state = M.prepare(wts, k)
    y, w, ids = M.forward(bf("x_bits"), state)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), f["ids"])
    c = om.compare(y, torch.from_numpy(f["y32"]))
    assert c["max_abs"] <= MAX_ABS and c["rel_fro"] <= REL_FRO, c


def test_zero_tokens():
    cfg = W.MoeConfig("z", 4, 128, 4, 128, 2)
    _, wts = _layer(cfg, 0)
    state = M.prepare(_to_dev(wts), 2)
    y, w, ids = M.forward(torch.empty((0, 128), dtype=torch.bfloat16, device="cuda"), state)
    torch.cuda.synchronize()
    assert y.shape == (0, 128) and ids.shape == (0, 2)


def test_pack_is_a_lossless_row_permutation():
    e, i, h = 3, 256, 64
    w = torch.randn((e, 2 * i, h), device="cuda").to(torch.bfloat16)
    p = M.pack_gate_up(w)
    torch.cuda.synchronize()
    idx = []
    for nb in range(i // 128):
        idx += list(range(nb * 128, nb * 128 + 128)) + list(range(i + nb * 128, i + nb * 128 + 128))
    assert torch.equal(p, w[:, idx, :])


def test_graph_capture_and_token_permutation_property():
    """The layer is graph-capturable (no host sync), deterministic, and permuting the tokens permutes
    the outputs bitwise (each token's rows are computed by the same tile math wherever they land)."""
    cfg = W.MoeConfig("g", 512, 512, 32, 256, 4, shared=1, shared_i=128)
    x, wts = _layer(cfg, 8)
    state = M.prepare(_to_dev(wts), cfg.k)
    gx = x.cuda()
    y0, w0, i0 = [t.clone() for t in M.forward(gx, state)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        M.forward(gx, state)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = M.forward(gx, state)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out[0], y0) and torch.equal(out[2], i0)
    perm = torch.randperm(cfg.t, generator=torch.Generator().manual_seed(1)).cuda()
    yp, wp, ip = M.forward(gx[perm].contiguous(), state)
    torch.cuda.synchronize()
    assert torch.equal(ip, i0[perm]) and torch.equal(yp, y0[perm]) and torch.equal(wp, w0[perm])


def test_prefill_full_size_properties():
    """MoE prefill configuration (T=8192, H=7168, 256 experts + shared, top-8), weights drawn on the
    GPU: routing of sampled tokens is bit-exact against the oracle; every expert count matches the
    ids; outputs are finite; token permutation property holds on a slice."""
    cfg = W.MOE_CONFIGS["moe_prefill"]
    gx = W.moe_input(cfg.t, cfg.h, 2, device="cuda")
    wts = W.moe_weights(cfg, 2, device="cuda")
    state = M.prepare(wts, cfg.k)
    del wts["w_gate_up"], wts["shared_gate_up"]
    y, w, ids = M.forward(gx, state)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y.float()).all())
    rows = torch.tensor([0, 1, 4095, 8191])
    olg = om.router_logits(gx[rows].cpu(), state["router"].cpu())
    oids, _ = om.topk(olg, cfg.k)
    assert torch.equal(ids[rows].cpu(), oids)
    assert torch.allclose(w[rows].cpu(), om.renorm_weights(olg, oids), atol=W_ATOL)
    p = M.plan(ids, w, cfg.e)
    torch.cuda.synchronize()
    assert torch.equal(p["counts"].cpu().long(), torch.bincount(ids.cpu().reshape(-1).long(), minlength=cfg.e))
    # one token's output against the oracle restricted to its own experts
    t = 4095
    xt = gx[t:t + 1].cpu()
    experts = oids[2].tolist()
    ref = torch.zeros(cfg.h)
    wt = w[t].cpu()
    for j, e in enumerate(experts):
        packed = state["w_gate_up_packed"][e].cpu()
        # undo the packing for the reference
        I = cfg.i
        idx = []
        for nb in range(I // 128):
            idx += list(range(nb * 256, nb * 256 + 128))
        gate = packed[idx]
        up = packed[[q + 128 for q in idx]]
        h = (torch.nn.functional.silu(gate.float() @ xt[0].float()) * (up.float() @ xt[0].float())).bfloat16().float()
        ref += wt[j] * (state["w_down"][e].cpu().float() @ h)
    sp = state["shared_gate_up_packed"][0].cpu()
    Is = cfg.shared_i
    idx = []
    for nb in range(Is // 128):
        idx += list(range(nb * 256, nb * 256 + 128))
    h = (torch.nn.functional.silu(sp[idx].float() @ xt[0].float()) *
         (sp[[q + 128 for q in idx]].float() @ xt[0].float())).bfloat16().float()
    ref += state["shared_down"][0].cpu().float() @ h
    c = om.compare(y[t:t + 1].cpu(), ref[None])
    assert c["max_abs"] <= MAX_ABS and c["rel_fro"] <= REL_FRO, c


# ------------------------------------------------------------------------------ tensor-core routing path
def _gamma(h: int) -> float:
    steps = (2 * h + 15) // 16
    return 2.0 ** -16 + 1.01 * 17.0 * 2.0 ** -23 * steps + 2.0 ** -20


@pytest.mark.parametrize("cfg", [
    W.MoeConfig("fast_small", 300, 512, 16, 128, 4),
    W.MoeConfig("fast_odd_e", 200, 640, 37, 128, 8),
    W.MoeConfig("fast_skew", 4096, 1024, 128, 128, 4, zipf_s=1.2),
    W.MoeConfig("fast_e256", 1024, 7168, 256, 128, 8),
    W.MoeConfig("fast_k32", 64, 256, 64, 128, 32),
])
def test_fast_route_equals_fixed_order_route(cfg):
    """ids and weights of the tensor-core path are bitwise those of the full fixed-order router."""
    x = W.moe_input(cfg.t, cfg.h, 5, device="cuda")
    router = W._randn((cfg.e, cfg.h), 77, "cuda", 1.0 / cfg.h ** 0.5, torch.float32)
    bias = W.zipf_router_bias(cfg.e, cfg.zipf_s, 5).cuda() if cfg.zipf_s > 0 else None
    lg, w0, i0 = M.route(x, router, bias, cfg.k)
    split, norms = M.prepare_router(router)
    w1, i1 = M.route_fast(x, router, bias, split, norms, cfg.k)
    torch.cuda.synchronize()
    assert torch.equal(i1, i0)
    assert torch.equal(w1.view(torch.int32), w0.view(torch.int32))
    rows = torch.arange(0, cfg.t, max(1, cfg.t // 16))
    olg = om.router_logits(x[rows].cpu(), router.cpu(), None if bias is None else bias.cpu())
    oids, _ = om.topk(olg, cfg.k)
    assert torch.equal(i1[rows].cpu(), oids)


def test_router_prepass_error_inside_bound():
    """Prefill-width router (H=7168, E=256): the tensor-core pre-pass stays far inside the bound the
    candidate selection relies on (the bound allows a worst-case accumulation; measured errors are
    orders of magnitude smaller)."""
    T, H, E = 2048, 7168, 256
    x = W.moe_input(T, H, 6, device="cuda")
    router = W._randn((E, H), 78, "cuda", 1.0 / H ** 0.5, torch.float32)
    split, norms = M.prepare_router(router)
    approx = M.router_approx(x, split)
    exact = (x.double() @ router.double().T)
    torch.cuda.synchronize()
    xn = x.double().norm(dim=1, keepdim=True)
    assert bool((norms.double() >= router.double().norm(dim=1)).all())
    delta = _gamma(H) * xn * norms.double().max() * 1.01
    ratio = float(((approx.double() - exact).abs() / delta).max())
    assert ratio < 0.05, ratio


def test_prefill_fast_and_exact_paths_agree():
    """The whole prefill routing (T=8192, E=256, H=7168): tensor-core path == fixed-order path."""
    cfg = W.MOE_CONFIGS["moe_prefill"]
    x = W.moe_input(cfg.t, cfg.h, 9, device="cuda")
    router = W._randn((cfg.e, cfg.h), 79, "cuda", 1.0 / cfg.h ** 0.5, torch.float32)
    _, w0, i0 = M.route(x, router, None, cfg.k)
    split, norms = M.prepare_router(router)
    w1, i1 = M.route_fast(x, router, None, split, norms, cfg.k)
    torch.cuda.synchronize()
    assert torch.equal(i1, i0) and torch.equal(w1, w0)


def test_sm_budget_leaves_results_unchanged():
    """kdb_set_sm_budget only resizes the persistent grids: the layer's output is bitwise the same."""
    from kdb200 import _lib as L
    cfg = W.MoeConfig("budget", 700, 512, 16, 256, 4, shared=1, shared_i=256)
    x = W.moe_input(cfg.t, cfg.h, 9, device="cuda")
    state = M.prepare(W.moe_weights(cfg, 9, device="cuda"), cfg.k)
    y0, w0, i0 = M.forward(x, state)
    prev = L.lib().kdb_set_sm_budget(37)
    try:
        assert L.lib().kdb_sm_budget() == 37
        y1, w1, i1 = M.forward(x, state)
    finally:
        L.lib().kdb_set_sm_budget(prev)
    torch.cuda.synchronize()
    assert L.lib().kdb_sm_budget() == prev
    assert torch.equal(y0, y1) and torch.equal(w0, w1) and torch.equal(i0, i1)


@pytest.mark.parametrize("cfg", [
    W.MoeConfig("fused_plain", 300, 512, 16, 256, 4),
    W.MoeConfig("fused_shared", 700, 1024, 32, 256, 8, shared=1, shared_i=256),
    W.MoeConfig("fused_skew", 2048, 512, 64, 128, 4, zipf_s=1.2),
    W.MoeConfig("fused_h384", 200, 384, 8, 128, 2, shared=1, shared_i=128),   # last pair tile half past H
])
def test_fused_combine_equals_stage_composition(cfg):
    """kdb_moe_expert_down_combine merges each token's slot rows in the down GEMM's epilogue (the last of the
    token's k tiles to arrive sums them in slot order).  Its rows and y must equal, bitwise, the separate
    stages: grouped down into per-slot rows, then the combine kernel; the layer (which uses the separate
    stages) agrees too."""
    x = W.moe_input(cfg.t, cfg.h, 21, device="cuda")
    state = M.prepare(W.moe_weights(cfg, 21, device="cuda"), cfg.k)
    y, w, ids = M.forward(x, state)
    p = M.plan(ids, w, cfg.e)
    mt = torch.zeros(cfg.e + 1, dtype=torch.int32, device="cuda")
    mt[1:] = torch.cumsum((p["counts"] + 511) // 512, 0)
    xp = M.gather_rows(x, p["perm_slot"], div=cfg.k)
    h = M.expert_gate_up(xp, state["w_gate_up_packed"], p["offsets"], mt)
    perm_w = w.reshape(-1)[p["perm_slot"].long()].contiguous()
    rows = M.expert_down(h, state["w_down"], p["offsets"], mt, perm_w)
    ys = None
    if cfg.shared:
        hs = M.expert_gate_up(x, state["shared_gate_up_packed"])
        ys = M.expert_down(hs, state["shared_down"])
    y2 = M.combine(rows, p["slot_pos"], cfg.t, cfg.k, shared_rows=ys)
    rows3, y3 = M.expert_down_combine(h, state["w_down"], p["offsets"], mt, perm_w, p["perm_slot"], p["slot_pos"],
                                      cfg.t, cfg.k, shared_rows=ys)
    rows4, y4 = M.expert_down_combine(h, state["w_down"], p["offsets"], mt, perm_w, p["perm_slot"], p["slot_pos"],
                                      cfg.t, cfg.k, shared_rows=ys)   # counters start from zero again
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    assert torch.equal(rows3, rows) and torch.equal(y3, y2) and torch.equal(y4, y2)
