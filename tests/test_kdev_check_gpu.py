"""The drop-in boundary on a GPU, driven by kdev itself: kdev's OKC adapter loads each real submission
(kernel-development_b200/submissions/b200_*.py) and its problem (oracle/problems/b200_*), and kdev's own
check path (`run_case`, src/kdev/checks/check.py:368-435) runs every test shape in eager mode, in CUDA-graph
mode (capture after a side-stream warm-up, replays compared bitwise with eager) and in graph_fresh mode (a
second seed's inputs copied into the captured buffers).  Every outcome must be "pass".

Reduced sizes keep the oracle's CPU check short: the MoE problems' configurations and the w4a16 problem's
are swapped for small ones with the same structure before kdev imports the problem references.  kdev comes
from $KDEV_SRC or from its offline install under baseline/_ref; without it the tests skip."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
KDEV_SRC = Path(os.environ["KDEV_SRC"]) if os.environ.get("KDEV_SRC") else ROOT / "baseline" / "_ref"
PROBLEMS = ROOT / "oracle" / "problems"
SUBS = ROOT / "kernel-development_b200" / "submissions"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (KDEV_SRC / "kdev" / "checks" / "check.py").exists(), reason="kdev not available")]


@pytest.fixture(scope="module")
def kdev():
    sys.path.insert(0, str(KDEV_SRC))
    try:
        from kdev.adapters import okc
        from kdev.checks import check
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"kdev not importable: {e}")
    yield okc, check
    sys.path.remove(str(KDEV_SRC))


def _fresh_references():
    for name in [n for n in list(sys.modules) if n.startswith("_kdev_ref_") or n == "moe_problem"]:
        del sys.modules[name]


def _run_all(okc, check, problem: str, submission: str, shapes=None):
    a = okc.OkcAdapter(str(PROBLEMS / problem), str(PROBLEMS / f"{problem}.toml"))
    mod = a.load(str(SUBS / submission), problem)
    state = a.prepare(mod)
    outcomes = []
    for shape in (shapes(a) if shapes else a.tests()):
        outcomes += check.run_case(a, mod, state, shape, 11, modes=("eager", "graph"), repeats=2, fresh_seed=12)
    bad = [(o.shape_id, o.mode, o.klass, o.message) for o in outcomes if o.klass != "pass"]
    assert not bad, bad
    modes = {o.mode for o in outcomes}
    assert {"eager", "graph", "graph_fresh"} <= modes, modes
    return outcomes


def test_projection_submission_passes_kdev_check(kdev):
    okc, check = kdev
    out = _run_all(okc, check, "b200_bf16_proj", "b200_bf16_proj.py",
                   shapes=lambda a: [s for s in a.tests() if s.case["m"] <= 4096])
    assert len({o.shape_id for o in out}) >= 5


@pytest.mark.parametrize("problem, small", [
    ("moe_decode", dict(t=64, h=512, e=16, i=256, k=4)),
    ("moe_prefill", dict(t=512, h=512, e=32, i=256, k=8, shared=1, shared_i=256)),
    ("moe_skewed", dict(t=1024, h=512, e=32, i=128, k=4, zipf_s=1.2)),
])
def test_moe_submissions_pass_kdev_check(kdev, monkeypatch, problem, small):
    okc, check = kdev
    sys.path.insert(0, str(ROOT / "kernel-development_b200"))
    from kdb200 import workloads as W
    monkeypatch.setitem(W.MOE_CONFIGS, problem, W.MoeConfig(problem, **small))
    _fresh_references()
    # the problem's tests plus its timing shape at the reduced width (more than 64 tokens per expert
    # group: the CTA-pair GEMMs with the combine fused into the down epilogue)
    _run_all(okc, check, f"b200_{problem}", f"b200_{problem}.py", shapes=lambda a: list(a.tests()) + list(a.shapes()))
    _fresh_references()


def test_w4a16_submission_passes_kdev_check(kdev, monkeypatch):
    okc, check = kdev
    sys.path.insert(0, str(ROOT / "kernel-development_b200"))
    from kdb200 import workloads as W
    monkeypatch.setitem(W.W4A16_CONFIGS, "w4a16_bs16", W.W4A16Config("w4a16_bs16", 16, 512, 256, 4, 32, 4))
    _fresh_references()
    _run_all(okc, check, "b200_moe_w4a16", "b200_moe_w4a16.py",
             shapes=lambda a: [s for s in a.tests() if s.case.get("bs", 0) <= 64])
    _fresh_references()
    torch.cuda.synchronize()


def test_attention_submission_passes_kdev_check(kdev):
    okc, check = kdev
    _run_all(okc, check, "b200_attention_decode", "b200_attention_decode.py",
             shapes=lambda a: [s for s in a.tests() if s.case["ctx"] <= 9000 and s.case["batch"] <= 8])
