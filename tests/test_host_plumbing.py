"""CPU tests of the Python layer's plumbing: well-formed calls, built the way prepare() / forward() and the
expert-parallel layer build them, pass every host-side check and reach the C entry point with the sizes the
header expects.  The device is faked (CPU tensors accepted as if on the GPU, a recording stub in place of
libkdb200), so nothing here launches a kernel; the GPU tests run the same calls for real."""
from __future__ import annotations

import contextlib
import importlib

import pytest
import torch

from kdb200 import _lib
from kdb200 import moe as M
from kdb200 import moe_w4a16 as W4
from kdb200 import workloads as W

P = importlib.import_module("kdb200.proj")        # the module (the package exports the op under this name)


class _Stub:
    """Records C calls; workspace-size queries return a small positive size, everything else status 0."""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def fn(*args):
            self.calls.append((name, args))
            return 4096 if name.endswith("workspace_bytes") else 0
        return fn


@pytest.fixture
def fake_device(monkeypatch):
    stub = _Stub()
    monkeypatch.setattr(_lib, "lib", lambda: stub)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())

    class _S:
        cuda_stream = 0
    monkeypatch.setattr(torch.cuda, "current_stream", lambda d=None: _S())
    return stub


def _names(stub):
    return [c[0] for c in stub.calls]


@pytest.mark.parametrize("cfg", [
    W.MoeConfig("plain", 6, 128, 8, 128, 2),
    W.MoeConfig("shared_bias", 5, 256, 16, 256, 4, shared=1, shared_i=128, zipf_s=1.2),
    W.MoeConfig("odd_h", 3, 72, 8, 128, 2),          # H % 64 != 0: no router split
])
def test_moe_prepare_and_forward_pass_checks(fake_device, cfg):
    state = M.prepare(W.moe_weights(cfg, 1), cfg.k)
    assert (state["router_split"] is None) == (cfg.h % 64 != 0)
    y, w, ids = M.forward(W.moe_input(cfg.t, cfg.h, 1), state)
    assert y.shape == (cfg.t, cfg.h) and w.shape == ids.shape == (cfg.t, cfg.k)
    name, args = fake_device.calls[-1]
    assert name == "kdb_moe_forward" and args[12:19] == (cfg.t, cfg.h, cfg.e, cfg.i, cfg.k, cfg.shared,
                                                          cfg.shared_i)


def test_expert_parallel_stages_pass_checks(fake_device):
    cfg = W.MoeConfig("ep", 8, 128, 8, 128, 2, shared=1, shared_i=128)
    state = M.prepare(W.moe_weights(cfg, 2), cfg.k)
    x = W.moe_input(cfg.t, cfg.h, 2)
    w, ids = M.route_fast(x, state["router"], None, state["router_split"], state["router_norms"], cfg.k)
    plan = M.plan(ids, w, cfg.e)
    send = M.gather_rows(x, plan["perm_slot"], div=cfg.k)
    counts = plan["counts"].view(2, cfg.e // 2)
    grouped, offsets, mtile = M.ep_regroup(counts, send, True)
    h = M.expert_gate_up(grouped, state["w_gate_up_packed"][: cfg.e // 2], offsets, mtile)
    yg = M.expert_down(h, state["w_down"][: cfg.e // 2], offsets, mtile)
    back, _, _ = M.ep_regroup(counts, yg, False)
    shared = M.expert_down(M.expert_gate_up(x, state["shared_gate_up_packed"][0:1]), state["shared_down"][0:1])
    M.combine(back, plan["slot_pos"], cfg.t, cfg.k, slot_w=w, shared_rows=shared)
    names = _names(fake_device)
    order = ["kdb_moe_route_fast", "kdb_moe_plan", "kdb_moe_gather_rows", "kdb_moe_ep_regroup",
             "kdb_moe_expert_gate_up", "kdb_moe_expert_down", "kdb_moe_ep_regroup", "kdb_moe_expert_gate_up",
             "kdb_moe_expert_down", "kdb_moe_combine"]
    pos = 0
    for n in names:                                  # the C calls happen in this order
        if pos < len(order) and n == order[pos]:
            pos += 1
    assert pos == len(order), names


def test_w4a16_forward_passes_checks(fake_device):
    cfg = W.W4A16Config("p", 5, 256, 128, 4, 32, 4)
    state = W4.prepare(W.w4a16_weights(cfg, 1), device="cpu")
    ids, tw = W.w4a16_routing(cfg, 1)
    y = W4.forward(W.moe_input(cfg.t, cfg.h, 1), ids.t().contiguous().t(), tw, state, cfg.e_total)
    assert y.shape == (cfg.t, cfg.h)
    name, args = fake_device.calls[-1]
    assert name == "kdb_moe_w4a16_forward" and args[9:15] == (cfg.t, cfg.h, cfg.i, cfg.local, cfg.e_total, cfg.k)


def test_projection_ops_pass_checks(fake_device):
    x = W.proj_input(16, 256, 1)
    y = P.proj(x, W.proj_weight(256, 512, 1))
    assert y.shape == (16, 512)
    split = P.split_f32(W.proj_weight_f32(256, 64, 1))
    assert split.shape == (64, 512) and split.dtype == torch.bfloat16
    y32 = P.proj_f32w(x, split)
    assert y32.shape == (16, 64) and y32.dtype == torch.float32
    assert _names(fake_device)[-1] == "kdb_proj_f32w"


@pytest.mark.parametrize("case", [dict(batch=2, ctx=300, heads="tp8", layer="sliding"),
                                  dict(batch=3, ctx=200, heads="dp", layer="full", q_len=8)])
def test_attention_decode_passes_checks(fake_device, case):
    from kdb200 import attention as A
    from oracle import attention as OA
    d = OA.generate_input(case, 3)
    out = A.decode(d["q"], d["k_new"], d["v_new"], d["k_cache"], d["v_cache"], d["block_table"], d["seq_lens"],
                   d["kv_scale"], A.window_of(case["layer"]))
    assert out.shape == d["q"].shape and out.dtype == torch.bfloat16
    name, args = fake_device.calls[-1]
    B, T, Hq, _ = d["q"].shape
    assert name == "kdb_attn_decode_fp8"
    assert args[7] == d["kv_scale"] and args[9:17] == (B, T, Hq, d["k_cache"].shape[1], 128,
                                                       d["block_table"].shape[1], d["k_cache"].shape[0],
                                                       A.window_of(case["layer"]))


def test_attention_decode_rejects_bad_arguments(fake_device):
    from kdb200 import attention as A
    from oracle import attention as OA
    d = OA.generate_input(dict(batch=1, ctx=50), 1)
    args = [d["q"], d["k_new"], d["v_new"], d["k_cache"], d["v_cache"], d["block_table"], d["seq_lens"]]
    with pytest.raises(TypeError):
        A.decode(d["q"].float(), *args[1:])
    with pytest.raises(TypeError):
        A.decode(*args[:3], d["k_cache"].view(torch.uint8), *args[4:])
    with pytest.raises(ValueError):
        A.decode(*args[:5], d["block_table"].repeat(2, 1), d["seq_lens"])
    with pytest.raises(ValueError):
        A.window_of("local")
