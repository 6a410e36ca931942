"""The drop-in boundary, exercised through kdev's own OKC adapter (CPU only).

kdev's OkcAdapter (src/kdev/adapters/okc.py:318-577) loads the problem dirs and TOMLs
(oracle/problems/) and a submission file, and calls prepare / make_inputs / call / check exactly as
`kdev check` does (src/kdev/checks/check.py:362-448).  The real submissions need a GPU, so the call
path uses a CPU stand-in with the same two entry points; the real submission files are loaded (not
called) to show they import cleanly through kdev's loader.  Skipped when kdev's sources are absent
($KDEV_SRC, else kdev's offline install under baseline/_ref)."""
from __future__ import annotations

import os
import sys
import textwrap
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
# kdev itself: $KDEV_SRC (a source tree's `src`), else its offline install under baseline/_ref
KDEV_SRC = Path(os.environ["KDEV_SRC"]) if os.environ.get("KDEV_SRC") else Path(__file__).resolve().parent.parent / "baseline" / "_ref"
PROBLEMS = ROOT / "oracle" / "problems"
SUBS = ROOT / "kernel-development_b200" / "submissions"

pytestmark = pytest.mark.skipif(not (KDEV_SRC / "kdev" / "adapters" / "okc.py").exists(),
                                reason="kdev sources not available")


@pytest.fixture(scope="module")
def okc():
    sys.path.insert(0, str(KDEV_SRC))
    try:
        from kdev.adapters import okc as mod
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"kdev not importable: {e}")
    yield mod
    sys.path.remove(str(KDEV_SRC))


CPU_PROJ_SUB = textwrap.dedent('''\
    # CPU stand-in with the submission's entry points (the real one launches libkdb200 kernels)
    import torch
    def prepare(weights):
        return {k: w.contiguous() for k, w in weights.items()}
    def kernel_fn(data, state):
        w = state[data["config"]["layer"]]
        y = data["x"].double() @ w.double().T
        return y.float() if w.dtype == torch.float32 else y.to(torch.bfloat16)
    ''')


def test_projection_problem_through_kdev(okc, tmp_path):
    a = okc.OkcAdapter(str(PROBLEMS / "b200_bf16_proj"), str(PROBLEMS / "b200_bf16_proj.toml"))
    assert a.problem == "b200_bf16_proj" and a.kernel_fn_args() == 2
    assert [s.shape_id for s in a.tests()] == ["t0", "t1", "t2", "t3", "t4", "t5", "t6"]
    assert any(s.case == {"m": 4096, "layer": "k7168_n7168"} for s in a.shapes())
    assert any(s.case.get("layer") == "router" for s in a.shapes())
    sub = tmp_path / "cpu_sub.py"
    sub.write_text(CPU_PROJ_SUB)
    mod = a.load(str(sub), "cpu")
    state = a.prepare(mod)
    for shape in [s for s in a.tests() if s.case["m"] <= 300]:
        data = a.make_inputs(shape, seed=7)
        out = a.call(mod, state, data)
        res = a.check(data, out)
        assert res.ok, (shape.shape_id, res.message)
        assert res.max_rel_err is not None and res.max_rel_err < 1e-2
        if shape.case["layer"] == "router":
            assert out.dtype == torch.float32 and res.tol == pytest.approx(1e-4)
            # a bf16 rounding of the fp32 router weights is outside the router layer's bound
            w16 = state["router"].to(torch.bfloat16).double()
            rough = (data["x"].double() @ w16.T).float()
            assert not a.check(data, rough).ok
        else:
            assert res.tol == pytest.approx(1e-2)
        bad = a.check(data, out * 1.5)
        assert not bad.ok
    m4096 = next(s for s in a.shapes() if s.shape_id == "m4096/k7168")
    sol = a.speed_of_light_us(m4096, {"hbm_bytes_per_s": 6.55e12, "bf16_dense_flops_per_s": 1.657e15})
    assert 200 < sol < 300      # 4096 x 7168 x 7168 at the measured bf16 peak


def test_real_submissions_load_through_kdev(okc):
    a = okc.OkcAdapter(str(PROBLEMS / "b200_bf16_proj"), str(PROBLEMS / "b200_bf16_proj.toml"))
    mod = a.load(str(SUBS / "b200_bf16_proj.py"), "real")
    assert callable(mod.prepare) and callable(mod.kernel_fn)
    for p in ("decode", "prefill", "skewed"):
        m = okc.OkcAdapter(str(PROBLEMS / f"b200_moe_{p}"), str(PROBLEMS / f"b200_moe_{p}.toml"))
        sm = m.load(str(SUBS / f"b200_moe_{p}.py"), f"real_{p}")
        assert callable(sm.prepare) and callable(sm.kernel_fn)


def test_moe_problem_check_through_kdev(okc, tmp_path, monkeypatch):
    """The decode MoE problem's reference checks an oracle-computed output as passing and a perturbed
    routing as failing, with kdev parsing the message."""
    sys.path.insert(0, str(ROOT))
    from kdb200 import workloads as W
    from oracle import moe as om
    small = W.MoeConfig("moe_decode", 64, 256, 16, 128, 4)
    monkeypatch.setitem(W.MOE_CONFIGS, "moe_decode", small)
    for name in [n for n in list(sys.modules) if n.startswith("_kdev_ref_")]:
        del sys.modules[name]
    a = okc.OkcAdapter(str(PROBLEMS / "b200_moe_decode"), str(PROBLEMS / "b200_moe_decode.toml"))
    w = a.weights()
    data = a.make_inputs(a.tests()[1], seed=3)
    ref = om.moe_ref(data["x"], w, small.k)
    res = a.check(data, (ref["y"], ref["w"], ref["ids"]))
    assert res.ok, res.message
    ids = ref["ids"].clone()
    ids[0, 0] = (ids[0, 0] + 1) % small.e
    res2 = a.check(data, (ref["y"], ref["w"], ids))
    assert not res2.ok and "mismatched 1" in res2.message


CPU_ATTN_SUB = textwrap.dedent('''\
    # CPU stand-in with the submission's entry point (the real one launches libkdb200 kernels)
    import sys
    sys.path.insert(0, ROOT)
    from oracle import attention as oa
    def kernel_fn(data):
        kc, vc = oa.append_kv(data)
        data["k_cache"].copy_(kc)
        data["v_cache"].copy_(vc)
        return oa.attention_ref(data).to(data["q"].dtype)
    ''')


def test_attention_problem_through_kdev(okc, tmp_path):
    """The attention problem (kernel_fn(data), check through collect): an oracle stand-in passes, an output
    off by 10 % fails, and a cache without the appended entries fails."""
    a = okc.OkcAdapter(str(PROBLEMS / "b200_attention_decode"), str(PROBLEMS / "b200_attention_decode.toml"))
    assert a.problem == "b200_attention_decode" and a.kernel_fn_args() == 1
    assert [s.shape_id for s in a.tests()][:3] == ["t0", "t1", "t2"]
    sub = tmp_path / "cpu_attn_sub.py"
    sub.write_text(CPU_ATTN_SUB.replace("ROOT", repr(str(ROOT))))
    mod = a.load(str(sub), "cpu_attn")
    shape = a.tests()[0]
    data = a.make_inputs(shape, seed=5)
    if data["q"].is_cuda:
        pytest.skip("CPU-only test")
    out = a.call(mod, None, data)
    res = a.check(data, out)
    assert res.ok, res.message
    assert not a.check(data, out * 1.1).ok
    fresh = a.make_inputs(shape, seed=5)
    bad = a.check(fresh, out)           # caches without the new entries
    assert not bad.ok and "k_cache" in bad.message
    real = a.load(str(SUBS / "b200_attention_decode.py"), "real_attn")
    assert callable(real.kernel_fn)
