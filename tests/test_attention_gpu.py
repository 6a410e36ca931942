"""GPU parity tests of the FP8-KV paged decode / verify attention (kdb_attn_decode_fp8) against the oracle
(oracle/attention.py): the cases of the reference's problem tests (okc_problems/muse_attention_decode.toml
[[tests]] t0-t15), edge lengths, both head layouts, q_len 1 and 8, sliding and full layers, kv_scale.

Tolerance (written here, the reference's check): relative L2 error of the output <= 2.5 x the error the
reference itself makes with FP8 E4M3 queries + 0.015.  The appended cache entries are compared bitwise with
the oracle's quantisation; every other cache byte must be unchanged."""
from __future__ import annotations

import pytest
import torch

from kdb200 import _lib
from kdb200 import attention as A
from oracle import attention as OA

pytestmark = pytest.mark.gpu


def _to_gpu(d):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def _run(case, seed=1, window=None):
    data = OA.generate_input(case, seed)
    layer = data["config"]["layer"]
    win = (OA.WINDOW if window is None else window) if layer == "sliding" else 0
    g = _to_gpu(data)
    out = A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"],
                   data["kv_scale"], win)
    torch.cuda.synchronize()
    return data, g, out


def _status():
    return _lib.status_read(torch.cuda.current_stream().cuda_stream)


def _check_cache(data, g):
    kc, vc = OA.append_kv(data)
    assert torch.equal(g["k_cache"].cpu().view(torch.uint8), kc.view(torch.uint8)), "k_cache differs"
    assert torch.equal(g["v_cache"].cpu().view(torch.uint8), vc.view(torch.uint8)), "v_cache differs"


TESTS = {   # the reference problem's [[tests]] cases (muse_attention_decode.toml)
    "t0": dict(batch=1, ctx=10, heads="tp8", layer="sliding"),
    "t1": dict(batch=3, ctx=2047, heads="tp8", layer="sliding"),
    "t2": dict(batch=5, ctx=5000, heads="tp8", layer="sliding", q_len=8, spread="mixed"),
    "t3": dict(batch=4, ctx=3000, heads="tp8", layer="full"),
    "t4": dict(batch=8, ctx=8192, heads="dp", layer="full", spread="mixed"),
    "t6": dict(batch=4, ctx=6000, heads="tp8", layer="sliding", dist="edges"),
    "t7": dict(batch=4, ctx=6000, heads="tp8", layer="full", q_len=8, dist="edges"),
    "t9": dict(batch=3, ctx=4000, heads="tp8", layer="sliding", q_len=8, kv_scale=0.015625),
    "t10": dict(batch=2, ctx=9000, heads="tp8", layer="full", kv_scale=0.015625),
    "t12": dict(batch=4, ctx=6000, heads="tp8", layer="sliding", q_len=8, dist="soft"),
    "t13": dict(batch=2, ctx=20000, heads="dp", layer="full", q_len=8, dist="soft"),
    "t15": dict(batch=2, ctx=20000, heads="dp", layer="full", q_len=8, dist="coherent"),
}


@pytest.mark.parametrize("name", list(TESTS))
def test_attention_matches_oracle_reference_tests(name):
    data, g, out = _run(TESTS[name], seed=100 + int(name[1:]))
    ok, msg = OA.check(data, out.cpu())
    assert ok, f"{name}: {msg}"
    _check_cache(data, g)
    assert _status()[0] == 0


@pytest.mark.parametrize("name, case", [
    ("t5", dict(batch=2, ctx=100000, heads="tp8", layer="full", q_len=8)),
    ("t11", dict(batch=4, ctx=80000, heads="tp8", layer="full", spread="mixed", dist="soft")),
    ("t14", dict(batch=4, ctx=80000, heads="tp8", layer="full", spread="mixed", dist="coherent")),
])
def test_attention_matches_oracle_long_contexts(name, case):
    data, g, out = _run(case, seed=100 + int(name[1:]))
    ok, msg = OA.check(data, out.cpu())
    assert ok, f"{name}: {msg}"
    assert _status()[0] == 0


@pytest.mark.parametrize("case, window", [
    (dict(batch=6, ctx=700, heads="tp8", layer="sliding", spread="mixed"), 300),      # window inside the context
    (dict(batch=3, ctx=500, heads="dp", layer="sliding", q_len=8, dist="edges"), 200),
    (dict(batch=2, ctx=129, heads="tp8", layer="full", q_len=8), None),               # tile + 1 keys
    (dict(batch=2, ctx=256, heads="dp", layer="full"), None),                          # exactly two tiles
    (dict(batch=3, ctx=8, heads="tp8", layer="full", q_len=8), None),                  # no cached keys
    (dict(batch=1, ctx=1, heads="tp8", layer="sliding"), None),                        # one key
    (dict(batch=48, ctx=3000, heads="tp8", layer="sliding", q_len=8, spread="agentic"), None),
    (dict(batch=16, ctx=9000, heads="tp8", layer="full", spread="agentic", dist="coherent"), None),
])
def test_attention_edge_lengths(case, window):
    data, g, out = _run(case, seed=7, window=window)
    ok, msg = OA.check(data, out.cpu(), window=window)
    assert ok, msg
    _check_cache(data, g)


@pytest.mark.parametrize("q_len", [2, 3, 5, 7])
@pytest.mark.parametrize("layer, heads, window", [("full", "tp8", None), ("sliding", "dp", 300)])
def test_attention_other_query_lengths(q_len, layer, heads, window):
    """Row counts between the problem's decode (8) and verify (64) shapes: 16 rows take the decode kernel with
    16 query columns, 24 / 40 / 56 rows the rows kernel with part of its 64-row block empty."""
    case = dict(batch=5, ctx=1500, heads=heads, layer=layer, q_len=q_len, spread="mixed")
    data, g, out = _run(case, seed=20 + q_len, window=window)
    ok, msg = OA.check(data, out.cpu(), window=window)
    assert ok, f"q_len {q_len}: {msg}"
    _check_cache(data, g)
    assert _status()[0] == 0


def test_attention_large_scores_rescale_path():
    """Keys late in each sequence score far above the earlier ones, so the running maximum rises by more
    than the lazy-rescale threshold mid-sequence and O is rescaled in tensor memory."""
    case = dict(batch=3, ctx=5000, heads="tp8", layer="full", q_len=8)
    data = OA.generate_input(case, 5)
    for b in range(3):
        L = int(data["seq_lens"][b])
        dirs = data["q"][b].float().reshape(8, 1, 8, 128).mean(dim=(0, 2))
        for k in range(9):                       # each about 5 log2 units above the one before
            sl = data["block_table"][b, int(L * (k + 1) / 10)].long()
            data["k_cache"][sl] = OA.quantize_kv(dirs / dirs.norm() * 30 * (k + 1), data["kv_scale"])
    g = _to_gpu(data)
    out = A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"],
                   data["kv_scale"], 0)
    ok, msg = OA.check(data, out.cpu())
    assert ok, msg


def test_attention_repeat_and_graph_replay_are_identical():
    data, g, out = _run(TESTS["t7"], seed=3)
    again = A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"],
                     data["kv_scale"], 0)
    assert torch.equal(out, again)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"],
                 data["kv_scale"], 0)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gout = A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"],
                        g["seq_lens"], data["kv_scale"], 0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, out)
    del graph


def test_attention_out_of_range_slot_is_reported():
    """A block-table entry past the cache is caught by the kernels' own bounds checks (status word,
    KDB_ERR_DEVICE_BOUNDS) instead of being read; the call itself still returns."""
    data = OA.generate_input(dict(batch=2, ctx=300, heads="tp8", layer="full"), 2)
    data["block_table"][1, 17] = data["k_cache"].shape[0] + 5
    g = _to_gpu(data)
    _status()
    A.decode(g["q"], g["k_new"], g["v_new"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"],
             data["kv_scale"], 0)
    st = _status()
    assert st[0] == _lib.KDB_ERR_DEVICE_BOUNDS and st[1] == 0x1AC


def test_attention_rejects_unsupported_shapes():
    data = OA.generate_input(dict(batch=1, ctx=40), 1)
    g = _to_gpu(data)
    q = g["q"].repeat(1, 9, 1, 1)                         # q_len 9 x 8 heads per KV head > 64 rows
    kn = g["k_new"].repeat(1, 9, 1, 1)
    bt = torch.arange(80, dtype=torch.int32, device="cuda").view(1, 80)
    sl = torch.tensor([49], dtype=torch.int32, device="cuda")
    kc = torch.zeros((80, 1, 128), dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(_lib.KdbError):
        A.decode(q, kn, kn.clone(), kc, kc.clone(), bt, sl, 1.0, 0)
