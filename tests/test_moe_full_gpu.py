"""GPU parity of the MoE layer at the full sizes of its benchmark configurations, by sampling.

* moe_prefill (T=8192, H=7168, 256 experts + shared, top-8): 256 tokens drawn across the batch are
  routed by the oracle (bit-exact ids and weights) and their outputs compared with the oracle's layer.
* moe_skewed (T=16384, H=4096, 128 experts, I=1536, top-4, Zipf(1.2) popularity): ids of every token
  equal the fixed-order router's; outputs of tokens routed to the hottest and to the coldest experts, and
  of random tokens, are compared with the oracle.  The hot experts hold thousands of tokens: several
  512-token chunks of one weight tile.
* The plain fp32 PyTorch router (softmax(x.float() @ Wr.T).topk) against the layer's routing on all
  three configurations: every token where they pick different experts must be a near-tie, i.e. the
  exact logits of the swapped experts differ by no more than the two fp32 logits' own rounding errors.

Tolerances: ids exact; routing weights within 1e-6 absolute; outputs within max-abs 2e-2 and relative
Frobenius 1e-2 of the fp32 oracle."""
from __future__ import annotations

import pytest
import torch

from kdb200 import moe as M
from kdb200 import workloads as W
from oracle import moe as om

pytestmark = pytest.mark.gpu
MAX_ABS = 2e-2
REL_FRO = 1e-2
W_ATOL = 1e-6


def _check_tokens(rows, gx, y, w, ids, wts, k):
    """Oracle layer on tokens `rows` (weights may live on the GPU: the oracle moves one expert at a time)."""
    xs = gx[rows].cpu()
    ref = om.moe_ref(xs, {**wts, "router": wts["router"].cpu(),
                          "router_bias": None if wts.get("router_bias") is None else wts["router_bias"].cpu()}, k)
    assert torch.equal(ids[rows].cpu(), ref["ids"]), "routing ids differ from the oracle"
    assert float((w[rows].cpu() - ref["w"]).abs().max()) <= W_ATOL
    c = om.compare(y[rows], ref["y32"])
    assert c["nonfinite"] == 0 and c["max_abs"] <= MAX_ABS and c["rel_fro"] <= REL_FRO, c
    ok, msg = om.check((y[rows], w[rows], ids[rows]), ref)
    assert ok, msg
    return c


def test_prefill_256_sampled_tokens_match_oracle():
    cfg = W.MOE_CONFIGS["moe_prefill"]
    gx = W.moe_input(cfg.t, cfg.h, 3, device="cuda")
    wts = W.moe_weights(cfg, 3, device="cuda")
    state = M.prepare(wts, cfg.k)
    y, w, ids = M.forward(gx, state)
    torch.cuda.synchronize()
    rows = torch.randperm(cfg.t, generator=torch.Generator().manual_seed(11))[:256].sort().values
    c = _check_tokens(rows, gx, y, w, ids, wts, cfg.k)
    hit = torch.unique(ids[rows.cuda()]).numel()
    assert hit >= 200, f"the sample reaches only {hit} experts"
    print(f"prefill: 256 tokens over {hit} experts: {c}")


def test_skewed_full_size():
    cfg = W.MOE_CONFIGS["moe_skewed"]
    gx = W.moe_input(cfg.t, cfg.h, 4, device="cuda")
    wts = W.moe_weights(cfg, 4, device="cuda")
    state = M.prepare(wts, cfg.k)
    y, w, ids = M.forward(gx, state)
    # every token's ids and weights against the full fixed-order router (bit-exact with the oracle's,
    # which the routing tests pin on golden files)
    _, w0, i0 = M.route(gx, wts["router"], wts["router_bias"], cfg.k)
    torch.cuda.synchronize()
    assert torch.equal(ids, i0) and torch.equal(w.view(torch.int32), w0.view(torch.int32))
    counts = torch.bincount(ids.reshape(-1).long(), minlength=cfg.e).cpu()
    hot = int(counts.argmax())
    live = (counts > 0).nonzero().flatten()
    cold = int(live[counts[live].argmin()])
    assert int(counts[hot]) > 4 * 512, f"hottest expert holds {int(counts[hot])} tokens"
    tok_hot = (ids == hot).any(dim=1).nonzero().flatten().cpu()
    tok_cold = (ids == cold).any(dim=1).nonzero().flatten().cpu()
    g = torch.Generator().manual_seed(12)
    pick = lambda t, n: t[torch.randperm(t.numel(), generator=g)[:n]]  # noqa: E731
    rows = torch.cat([pick(tok_hot, 128), pick(tok_cold, 64),
                      torch.randperm(cfg.t, generator=g)[:64]]).unique().sort().values
    c = _check_tokens(rows, gx, y, w, ids, wts, cfg.k)
    print(f"skewed: hottest expert {hot} ({int(counts[hot])} tokens), coldest {cold} ({int(counts[cold])}); "
          f"{rows.numel()} tokens: {c}")


@pytest.mark.parametrize("name", ["moe_decode", "moe_prefill", "moe_skewed"])
def test_plain_fp32_router_differs_only_at_near_ties(name):
    """The layer routes on correctly rounded logits (fixed-order fp64 sums).  A plain fp32 PyTorch
    router on the host, softmax(x.float() @ Wr.T (+ b)).topk(k), can only pick a different expert e'
    over e (exact(e) > exact(e')) if its own logit errors err = fp32 - exact make up the gap:
    exact(e) - exact(e') <= |err(e)| + |err(e')| (+ softmax rounding).  Every differing token must
    satisfy that; the count is printed."""
    cfg = W.MOE_CONFIGS[name]
    x = W.moe_input(cfg.t, cfg.h, 1, device="cuda")
    router = W._randn((cfg.e, cfg.h), 1 * 1000 + 3, "cuda", 1.0 / cfg.h ** 0.5, torch.float32)
    bias = W.zipf_router_bias(cfg.e, cfg.zipf_s, 1).cuda() if cfg.zipf_s > 0 else None
    split, norms = M.prepare_router(router)
    w_ours, ids_ours = M.route_fast(x, router, bias, split, norms, cfg.k)
    exact = x.double() @ router.double().T          # bf16 x fp32 products are exact in fp64
    if bias is not None:
        exact = exact + bias.double()
    torch.cuda.synchronize()
    lg32 = om.torch_fp32_logits(x.cpu(), router.cpu(), None if bias is None else bias.cpu())
    ids_ref = torch.topk(torch.softmax(lg32, dim=-1), cfg.k, dim=-1).indices
    ex = exact.cpu()
    err = (lg32.double() - ex).abs()
    ours = ids_ours.cpu().long()
    diff_tokens = []
    for t in range(cfg.t):
        a, b = set(ours[t].tolist()), set(ids_ref[t].tolist())
        if a == b:
            continue
        diff_tokens.append(t)
        for e in a - b:
            for e2 in b - a:
                gap = float(ex[t, e] - ex[t, e2])
                slack = float(err[t, e] + err[t, e2]) + 4e-7 * max(1.0, abs(float(ex[t, e])))
                assert gap <= slack, (t, e, e2, gap, slack)
    max_err = float(err.max())
    print(f"{name}: {len(diff_tokens)} of {cfg.t} tokens route differently under the plain fp32 router "
          f"(all near-ties); max |fp32 logit - exact| = {max_err:.3e}")
    assert len(diff_tokens) <= max(2, cfg.t // 500)
