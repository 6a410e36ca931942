"""CPU tests of the oracle itself: the C routing restatement against independent numpy
restatements, the fp32 layer restatement against a per-token loop, and the golden fixtures."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from kdb200 import workloads as W
from oracle import moe as om
from oracle import proj as op

GOLDEN = Path(__file__).resolve().parent / "golden"


def _canon_logits_np(x: torch.Tensor, w: torch.Tensor) -> np.ndarray:
    """The fixed fp64 order of routing.c written with numpy arrays: 32 partials, partial l taking
    h = 256*b + 8*l + j (j = 0..7) block by block (products of bf16 x fp32 are exact in fp64, so
    a*b + c is one rounding like fma), then the xor butterfly 16, 8, 4, 2, 1, then one rounding
    to fp32."""
    xd = x.float().double().numpy()
    wd = w.double().numpy()
    T, H = xd.shape
    E = wd.shape[0]
    acc = np.zeros((T, E, 32))
    lanes = np.arange(32)
    for base in range(0, H, 256):
        for j in range(8):
            hs = base + 8 * lanes + j
            ok = hs < H
            acc[:, :, ok] = acc[:, :, ok] + xd[:, None, hs[ok]] * wd[None, :, hs[ok]]
    for off in (16, 8, 4, 2, 1):
        acc = acc + acc[:, :, lanes ^ off]
    return acc[:, :, 0].astype(np.float32)


@pytest.mark.parametrize("T,H,E", [(5, 64, 8), (17, 520, 33), (3, 7, 5), (8, 4096, 64), (4, 300, 9)])
def test_router_logits_fixed_order(T, H, E):
    g = torch.Generator().manual_seed(T * 131 + H)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    w = torch.randn((E, H), generator=g) / H ** 0.5
    got = om.router_logits(x, w).numpy()
    want = _canon_logits_np(x, w)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # and it is the correctly rounded dot product except, rarely, by one ulp
    exact = (x.double() @ w.double().T).numpy().astype(np.float32)
    ulps = np.abs(got.view(np.int32).astype(np.int64) - exact.view(np.int32).astype(np.int64))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3


def test_router_bias_is_one_fp32_add():
    g = torch.Generator().manual_seed(5)
    x = torch.randn((4, 96), generator=g).to(torch.bfloat16)
    w = torch.randn((6, 96), generator=g)
    b = torch.randn(6, generator=g)
    l0 = om.router_logits(x, w)
    l1 = om.router_logits(x, w, b)
    assert torch.equal(l1, (l0 + b).float())


def test_topk_matches_stable_sort_and_ties():
    g = torch.Generator().manual_seed(1)
    lg = torch.randn((50, 37), generator=g)
    lg[3, :] = 0.5                      # all tied: lower expert first
    lg[7, 10] = lg[7, 20] = lg[7].max() + 1
    ids, vals = om.topk(lg, 6)
    order = np.argsort(-lg.numpy(), axis=1, kind="stable")[:, :6]
    assert np.array_equal(ids.numpy(), order.astype(np.int32))
    assert ids[3].tolist() == [0, 1, 2, 3, 4, 5]
    assert ids[7, :2].tolist() == [10, 20]
    assert torch.equal(vals, lg.gather(1, ids.long()))


def test_permute_matches_lexsort():
    g = torch.Generator().manual_seed(2)
    T, k, E = 300, 4, 23
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    p = om.permute(ids, E)
    flat = ids.reshape(-1).numpy()
    slots = np.arange(T * k)
    order = np.lexsort((slots, flat))         # expert major, slot (hence token) minor
    assert np.array_equal(p["perm_slot"].numpy(), order.astype(np.int32))
    assert np.array_equal(p["counts"].numpy(), np.bincount(flat, minlength=E).astype(np.int32))
    assert p["offsets"][0] == 0 and p["offsets"][-1] == T * k
    inv = np.empty_like(order)
    inv[order] = np.arange(T * k)
    assert np.array_equal(p["slot_pos"].numpy(), inv.astype(np.int32))


def test_permute_rejects_bad_id():
    ids = torch.tensor([[0, 5]], dtype=torch.int32)
    with pytest.raises(ValueError):
        om.permute(ids, 4)


def test_renorm_weights_equal_softmax_over_picks():
    g = torch.Generator().manual_seed(3)
    lg = torch.randn((20, 16), generator=g)
    ids, vals = om.topk(lg, 4)
    w = om.renorm_weights(lg, ids)
    alt = torch.softmax(vals.double(), dim=-1).float()
    assert torch.allclose(w, alt, rtol=1e-6, atol=1e-7)
    assert torch.allclose(w.sum(-1), torch.ones(20), atol=1e-6)


def _naive_moe(x, wts, k):
    """Per-token loop restatement of the layer (independent of moe_ref's grouping)."""
    lg, ids, w = om.route(x, wts["router"], wts.get("router_bias"), k)
    T, H = x.shape
    I = wts["w_gate_up"].shape[1] // 2
    out = torch.zeros((T, H))
    for t in range(T):
        xt = x[t].float()
        for j in range(k):
            e = int(ids[t, j])
            gu = wts["w_gate_up"][e].float()
            h = (torch.nn.functional.silu(gu[:I] @ xt) * (gu[I:] @ xt)).bfloat16().float()
            out[t] += w[t, j] * (wts["w_down"][e].float() @ h)
        if wts.get("shared_gate_up") is not None:
            gu = wts["shared_gate_up"][0].float()
            Is = gu.shape[0] // 2
            h = (torch.nn.functional.silu(gu[:Is] @ xt) * (gu[Is:] @ xt)).bfloat16().float()
            out[t] += wts["shared_down"][0].float() @ h
    return out


@pytest.mark.parametrize("shared", [0, 1])
def test_moe_ref_matches_per_token_loop(shared):
    cfg = W.MoeConfig("t", 12, 64, 8, 128, 3, shared=shared, shared_i=128 if shared else 0)
    x = W.moe_input(cfg.t, cfg.h, 4)
    wts = W.moe_weights(cfg, 4)
    ref = om.moe_ref(x, wts, cfg.k)
    naive = _naive_moe(x, wts, cfg.k)
    assert torch.allclose(ref["y32"], naive, rtol=1e-5, atol=1e-5)


def test_check_messages_parse_like_kdev():
    """Check messages carry 'relative L2 error X (worst row Y) ... [bound B' as kdev's
    parse_check_message expects (src/kdev/adapters/okc.py:231-247)."""
    import re
    ok, msg = op.check(torch.ones(2, 3), torch.ones(2, 3))
    assert ok
    f = r"([0-9.]+(?:e[+-]?\d+)?)"
    assert re.search(r"relative L2 error " + f, msg)
    assert re.search(r"\[bound " + f, msg)
    assert re.search(r"worst row " + f, msg)
    bad, msg2 = op.check(torch.ones(2, 3) * 2, torch.ones(2, 3))
    assert not bad


def test_moe_check_reports_the_worst_token_row():
    """The MoE check's "(worst row Y)" is the largest per-token relative L2 error, not the overall one: a
    mistake planted in one token's output row of the oracle's own result shows up there alone."""
    import re
    cfg = W.MoeConfig("worst", 12, 64, 4, 128, 2)
    x = W.moe_input(cfg.t, cfg.h, 5)
    wts = W.moe_weights(cfg, 5)
    ref = om.moe_ref(x, wts, cfg.k)
    y = ref["y32"].clone()
    y[7] *= 1.015                                      # 1.5 % on one token only
    _, msg = om.check((y.bfloat16(), ref["w"], ref["ids"]), ref)
    f = r"([0-9.]+(?:e[+-]?\d+)?)"
    overall = float(re.search(r"relative L2 error " + f, msg).group(1))
    worst = float(re.search(r"worst row " + f, msg).group(1))
    assert 1.2e-2 < worst < 1.8e-2 and worst > 2 * overall, msg


def test_zipf_bias_fits_exponent():
    tau, s_fit = W.zipf_tau(128, 1.2)
    assert 0.1 < tau < 2.0
    assert abs(s_fit - 1.2) < 0.05
    b = W.zipf_router_bias(128, 1.2, seed=0)
    assert b.shape == (128,) and float(b.max()) == 0.0


# ------------------------------------------------------------------------------------ golden fixtures
def _manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())


def test_golden_files_hash():
    man = _manifest()
    assert man["files"], "empty manifest"
    for name, digest in man["files"].items():
        data = (GOLDEN / name).read_bytes()
        assert hashlib.sha256(data).hexdigest() == digest, name


def test_golden_routing_reproduces():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    for case in mg.ROUTING_CASES:
        f = np.load(GOLDEN / f"{case['name']}.npz")
        x, wts = mg.routing_inputs(case)
        lg = om.router_logits(x, wts["router"], wts["router_bias"])
        assert np.array_equal(lg.numpy().view(np.uint32), f["logits"].view(np.uint32)), case["name"]
        ids, _ = om.topk(lg, case["k"])
        assert np.array_equal(ids.numpy(), f["ids"]), case["name"]
        p = om.permute(ids, case["e"])
        assert np.array_equal(p["perm_slot"].numpy(), f["perm_slot"]), case["name"]


def test_golden_layer_reproduces():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    for case in mg.LAYER_CASES:
        f = np.load(GOLDEN / f"{case['name']}.npz")
        x, wts, cfg = mg.layer_inputs(case)
        ref = om.moe_ref(x, wts, cfg.k)
        assert np.array_equal(ref["ids"].numpy(), f["ids"])
        assert np.allclose(ref["y32"].numpy(), f["y32"], rtol=1e-5, atol=1e-6)
    for case in mg.PROJ_CASES:
        f = np.load(GOLDEN / f"{case['name']}.npz")
        x, w = mg.proj_inputs(case)
        assert np.allclose(op.proj_ref(x, w).numpy(), f["y32"], rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------------------ NVFP4 (w4a16) oracle
def test_nvfp4_codes_and_dequant_are_exact():
    from kdb200 import workloads as W
    vals = torch.tensor(W.E2M1_VALUES + tuple(-v for v in W.E2M1_VALUES[1:]))
    assert torch.equal(W.e2m1_decode(W.e2m1_encode(vals)), vals)          # every representable value round-trips
    w = torch.randn(256, 512) / 20
    q, s, g = W.nvfp4_quantize(w)
    dq = W.nvfp4_dequantize(q, s)
    assert torch.equal(dq, dq.to(torch.bfloat16).float())                  # e2m1 * e4m3 is exact in bf16
    assert torch.equal(dq, dq.to(torch.float16).float())                   # and in f16 (the kernel's operand)
    rel = float(((dq * g) - w).norm() / w.norm())
    assert rel < 0.12                                                      # 4-bit quantisation error


def test_e2m1_encoder_is_nearest_with_ties_to_even():
    from kdb200 import workloads as W
    grid = torch.tensor(W.E2M1_VALUES)
    mids = (grid[1:] + grid[:-1]) / 2
    v = torch.cat([torch.randn(20000) * 3, mids, -mids, grid, -grid, torch.tensor([7.0, -7.0, 1e-30, -1e-30])])
    codes = W.e2m1_encode(v)
    # brute force: nearest magnitude, exact ties to the even index (mantissa bit 0), saturation at 6
    mag = v.abs().clamp(max=6.0)
    d = (mag.unsqueeze(-1) - grid).abs()
    best = d.min(-1, keepdim=True).values
    cand = d == best
    even = cand & (torch.arange(8) % 2 == 0)
    idx = torch.where(even.any(-1), even.float().argmax(-1), cand.float().argmax(-1))
    want = (((v < 0) & (idx > 0)).to(torch.uint8) << 3) | idx.to(torch.uint8)
    assert torch.equal(codes, want)


def test_w4a16_expert_subset_equals_full_set():
    from kdb200 import workloads as W
    cfg = W.W4A16Config("sub", 2, 256, 128, 4, 32, 2)
    full = W.w4a16_weights(cfg, 3)
    sub = W.w4a16_weights(cfg, 3, experts=[2, 0])
    for k in ("w13", "w2", "w13_gscale", "w2_gscale"):
        assert torch.equal(sub[k][0], full[k][2]) and torch.equal(sub[k][1], full[k][0])
    assert torch.equal(sub["w13_scale"][0].view(torch.uint8), full["w13_scale"][2].view(torch.uint8))


def test_w4a16_oracle_skips_remote_routes_and_normalises():
    from kdb200 import workloads as W
    from oracle import moe_w4a16 as ow
    cfg = W.W4A16Config("t", 6, 128, 128, 2, 16, 3)
    wts = W.w4a16_weights(cfg, 4)
    x = W.moe_input(cfg.t, cfg.h, 4)
    ids = torch.tensor([[0, 5, 9], [1, 0, 7], [8, 9, 10], [1, 2, 3], [0, 1, 15], [4, 4, 4]], dtype=torch.int32)
    tw = torch.full((6, 3), 1.0 / 3)
    out = ow.w4a16_ref(x, ids, tw, wts, cfg.local)
    assert float(out[2].abs().max()) == 0.0 and float(out[5].abs().max()) == 0.0   # no local routes
    # one local route: the output row is tw * y / rms(y), whose RMS is tw (up to the 1e-8 and bf16 of y)
    rms = float((out[0] ** 2).mean().sqrt())
    assert abs(rms - 1.0 / 3) < 1e-3


def test_w4a16_blocks_are_a_permutation():
    from kdb200 import workloads as W
    import importlib
    W4 = importlib.import_module("kdb200.moe_w4a16")
    cfg = W.W4A16Config("t", 2, 256, 256, 2, 16, 2)
    wts = W.w4a16_weights(cfg, 1)
    I = cfg.i
    b13 = W4._blocks(wts["w13"], wts["w13_scale"], gate_up=True)            # [L, I/128, H/64, 9216]
    assert tuple(b13.shape) == (2, I // 128, cfg.h // 64, 9216)
    # tile f=1, chunk 2: part 0 row 5 = gate row 128 + 5, part 1 row 5 = up row I + 128 + 5
    blk = b13[1, 1, 2]
    assert torch.equal(blk[5 * 32:6 * 32], wts["w13"][1, 128 + 5, 64:96])
    assert torch.equal(blk[4096 + 5 * 32:4096 + 6 * 32], wts["w13"][1, I + 128 + 5, 64:96])
    assert torch.equal(blk[8192 + 512 + 7 * 4:8192 + 512 + 8 * 4], wts["w13_scale"][1, I + 128 + 7, 8:12].view(torch.uint8))
    b2 = W4._blocks(wts["w2"], wts["w2_scale"], gate_up=False)               # [L, H/256, I/64, 9216]
    blk2 = b2[0, 0, 1]
    assert torch.equal(blk2[4096 + 3 * 32:4096 + 4 * 32], wts["w2"][0, 128 + 3, 32:64])
    n = wts["w13"].numel() + wts["w13_scale"].numel()
    assert b13.numel() == n and sorted(b13.flatten().tolist()) == sorted(
        torch.cat([wts["w13"].flatten(), wts["w13_scale"].view(torch.uint8).flatten()]).tolist())


def test_projection_check_scales_max_abs_with_output_rms():
    """Unit-scale outputs keep the 2e-2 max-abs bound; heavy-tailed inputs (the outliers distribution) scale it
    with rms(Y), so a bf16-rounded result passes and a 1 % error still fails."""
    from kdb200 import workloads as W
    x = W.proj_input(64, 512, 3, dist="outliers")
    w = W.proj_weight(512, 256, 3)
    ref = op.proj_ref(x, w)
    assert float(ref.pow(2).mean().sqrt()) > 4
    ok, msg = op.check(ref.bfloat16(), ref)
    assert ok, msg
    bad, _ = op.check((ref * 1.02).bfloat16(), ref)
    assert not bad
    x1 = W.proj_input(64, 512, 3)
    ref1 = op.proj_ref(x1, w)
    assert abs(op.max_abs_bound(ref1) - op.MAX_ABS_TOL) < 1e-2 * op.MAX_ABS_TOL or op.max_abs_bound(ref1) <= 0.021
