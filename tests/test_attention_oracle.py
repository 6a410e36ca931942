"""CPU tests of the fp8-KV decode/verify attention oracle (oracle/attention.py): a naive per-query loop,
window and causality semantics, the cache append, and the check's message and bound."""
from __future__ import annotations

import math
import re

import pytest
import torch

from oracle import attention as A


def _naive(data, window):
    kc, vc = A.append_kv(data)
    q = data["q"].float()
    B, T, Hq, D = q.shape
    Hkv = kc.shape[1]
    out = torch.zeros((B, T, Hq, D))
    for b in range(B):
        L = int(data["seq_lens"][b])
        for t in range(T):
            p = L - T + t
            lo = max(0, p - window + 1) if data["config"]["layer"] == "sliding" else 0
            for h in range(Hq):
                g = h // (Hq // Hkv)
                sl = data["block_table"][b, lo:p + 1].long()
                K = kc[sl, g].float() * data["kv_scale"]
                V = vc[sl, g].float() * data["kv_scale"]
                a = torch.softmax(K @ q[b, t, h] / math.sqrt(D), dim=0)
                out[b, t, h] = a @ V
    return out


@pytest.mark.parametrize("case", [
    {"batch": 2, "ctx": 40, "heads": "tp8", "layer": "full"},
    {"batch": 3, "ctx": 50, "heads": "tp8", "layer": "sliding", "q_len": 8, "spread": "mixed"},
    {"batch": 2, "ctx": 30, "heads": "dp", "layer": "sliding", "dist": "edges", "kv_scale": 0.015625},
    {"batch": 4, "ctx": 64, "heads": "tp8", "layer": "full", "q_len": 8, "spread": "agentic", "dist": "coherent"},
])
def test_oracle_equals_naive_loop(case):
    data = A.generate_input(case, seed=11)
    win = 16
    got = A.attention_ref(data, window=win)
    want = _naive(data, win)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-4)


def test_sliding_window_ignores_older_keys():
    case = {"batch": 1, "ctx": 60, "layer": "sliding", "q_len": 1}
    data = A.generate_input(case, seed=3)
    base = A.attention_ref(data, window=20)
    L = int(data["seq_lens"][0])
    old = data["block_table"][0, :L - 20].long()                 # keys outside every query's window
    data["k_cache"][old] = A.quantize_kv(torch.randn(old.numel(), 1, A.HEAD_DIM) * 50, data["kv_scale"])
    assert torch.equal(A.attention_ref(data, window=20), base)
    data["config"]["layer"] = "full"
    assert not torch.equal(A.attention_ref(data, window=20), base)   # a full layer sees them


def test_verify_queries_are_causal():
    data = A.generate_input({"batch": 1, "ctx": 30, "q_len": 8}, seed=4)
    base = A.attention_ref(data)
    data["k_new"][0, 7] = data["k_new"][0, 7] * 3 + 1            # the last new token's key
    out = A.attention_ref(data)
    assert torch.equal(out[0, :7], base[0, :7]) and not torch.equal(out[0, 7], base[0, 7])


def test_append_writes_fp8_of_the_new_entries():
    data = A.generate_input({"batch": 2, "ctx": 20, "q_len": 8, "kv_scale": 0.015625}, seed=5)
    kc, vc = A.append_kv(data)
    for b in range(2):
        L = int(data["seq_lens"][b])
        sl = data["block_table"][b, L - 8:L].long()
        assert torch.equal(kc[sl].view(torch.uint8), A.quantize_kv(data["k_new"][b], 0.015625).view(torch.uint8))
        assert torch.equal(vc[sl].view(torch.uint8), A.quantize_kv(data["v_new"][b], 0.015625).view(torch.uint8))
        assert not bool((data["k_cache"][sl].float() != 0).any())     # reserved, not written, before the call


def test_gqa_heads_of_a_group_share_keys():
    data = A.generate_input({"batch": 1, "ctx": 25, "heads": "tp8"}, seed=6)
    data["q"][0, 0, 3] = data["q"][0, 0, 0]
    out = A.attention_ref(data)
    assert torch.equal(out[0, 0, 3], out[0, 0, 0])


def test_check_message_and_bound():
    data = A.generate_input({"batch": 2, "ctx": 300, "q_len": 8, "layer": "sliding"}, seed=7)
    ref = A.attention_ref(data)
    ok, msg = A.check(data, ref.to(torch.bfloat16))
    assert ok
    f = r"([0-9.]+(?:e[+-]?\d+)?)"
    m = re.search(r"relative L2 error " + f + r" \(worst row " + f + r"\) \[bound " + f, msg)
    assert m and float(m.group(1)) < 0.01
    yard = float(re.search(r"the reference's " + f, msg).group(1))
    assert abs(float(m.group(3)) - (2.5 * yard + 0.015)) < 2e-3
    bad, _ = A.check(data, torch.zeros_like(ref))
    assert not bad


def test_case_fields_and_lengths():
    c = A.AttnCase.from_dict({"batch": 16, "ctx": 80000, "heads": "tp8", "layer": "full", "page": 1,
                              "spread": "agentic", "dist": "coherent", "seed": 1})
    assert (c.q_heads, c.kv_heads) == (8, 1)
    lens = A.seq_lens(c, torch.Generator().manual_seed(0))
    assert int(lens[0]) == 80000 and bool((lens >= 5000).all()) and bool((lens <= 80000).all())


# Case fields of the reference's own attention tests (muse_attention_decode.toml [[tests]] t0-t7, t9, t10,
# t12, t13, t15); the ctx = 80k and 1M cases are left to the GPU.
REFERENCE_TEST_CASES = {
    "t0": {"batch": 1, "ctx": 10, "heads": "tp8", "layer": "sliding"},
    "t1": {"batch": 3, "ctx": 2047, "heads": "tp8", "layer": "sliding"},
    "t2": {"batch": 5, "ctx": 5000, "heads": "tp8", "layer": "sliding", "q_len": 8, "spread": "mixed", "page": 1},
    "t3": {"batch": 4, "ctx": 3000, "heads": "tp8", "layer": "full"},
    "t4": {"batch": 8, "ctx": 8192, "heads": "dp", "layer": "full", "spread": "mixed"},
    "t6": {"batch": 4, "ctx": 6000, "heads": "tp8", "layer": "sliding", "dist": "edges", "page": 1},
    "t7": {"batch": 4, "ctx": 6000, "heads": "tp8", "layer": "full", "q_len": 8, "dist": "edges"},
    "t9": {"batch": 3, "ctx": 4000, "heads": "tp8", "layer": "sliding", "q_len": 8, "page": 1, "kv_scale": 0.015625},
    "t10": {"batch": 2, "ctx": 9000, "heads": "tp8", "layer": "full", "kv_scale": 0.015625},
    "t12": {"batch": 4, "ctx": 6000, "heads": "tp8", "layer": "sliding", "q_len": 8, "dist": "soft", "page": 1},
    "t13": {"batch": 2, "ctx": 20000, "heads": "dp", "layer": "full", "q_len": 8, "dist": "soft"},
    "t15": {"batch": 2, "ctx": 20000, "heads": "dp", "layer": "full", "q_len": 8, "dist": "coherent"},
}


@pytest.mark.parametrize("name", sorted(REFERENCE_TEST_CASES))
def test_reference_test_shapes_run_and_check(name):
    case = REFERENCE_TEST_CASES[name]
    data = A.generate_input(case, seed=100 + len(name))
    c = A.AttnCase.from_dict(case)
    assert data["q"].shape == (c.batch, c.q_len, c.q_heads, A.HEAD_DIM)
    assert data["k_cache"].dtype == torch.float8_e4m3fn and int(data["seq_lens"].max()) <= c.ctx
    ref = A.attention_ref(data)
    assert bool(torch.isfinite(ref).all())
    ok, msg = A.check(data, ref.to(torch.bfloat16))
    assert ok, msg
