"""CPU tests of the Python layer's argument checks: the ops hand raw pointers to the kernels, so a wrong
dtype, shape or device must raise on the host before anything is launched."""
from __future__ import annotations

import pytest
import torch

from kdb200 import moe_w4a16 as W4
from kdb200 import workloads as W


def _w4_args(t=5, h=256, i=128, local=4, k=4):
    cfg = W.W4A16Config("chk", t, h, i, local, 32, k)
    st = W4.prepare(W.w4a16_weights(cfg, 1), device="cpu")
    x = torch.zeros((t, h), dtype=torch.bfloat16)
    ids = torch.zeros((t, k), dtype=torch.int32)
    tw = torch.full((t, k), 1.0 / k)
    return [x, ids, tw, st["w13_blocks"], st["w13_gscale"], st["w2_blocks"], st["w2_gscale"], st["pw1"], 32]


def test_w4a16_prepare_shapes_on_cpu():
    a = _w4_args()
    assert tuple(a[3].shape) == (4, 1, 4, 9216) and a[3].dtype == torch.uint8     # 2I/256 tiles, H/64 chunks
    assert tuple(a[5].shape) == (4, 1, 2, 9216)                                     # H/256 tiles, I/64 chunks
    assert tuple(a[4].shape) == (4,) and a[4].dtype == torch.float32


@pytest.mark.parametrize("pos, bad, exc", [
    (0, torch.zeros((5, 256), dtype=torch.float16), TypeError),          # x not bf16
    (1, torch.zeros((5, 4), dtype=torch.int64), TypeError),             # ids not int32
    (2, torch.zeros((5, 4), dtype=torch.float64), TypeError),           # weights not fp32
    (3, torch.zeros((4, 1, 4, 9216), dtype=torch.int8), TypeError),     # blocks not uint8
    (4, torch.zeros(4, dtype=torch.float16), TypeError),                # global scales not fp32
    (1, torch.zeros((5, 3), dtype=torch.int32), ValueError),            # ids / weights shapes differ
    (1, torch.zeros((6, 4), dtype=torch.int32), ValueError),            # ids rows != tokens
    (5, torch.zeros((4, 1, 3, 9216), dtype=torch.uint8), ValueError),   # down blocks for another I
    (6, torch.zeros(3, dtype=torch.float32), ValueError),               # one scale per local expert
    (7, torch.ones(128, dtype=torch.float32), ValueError),              # pw1 is one weight per hidden feature
    (7, torch.ones(256, dtype=torch.float16), ValueError),              # pw1 not fp32
    (8, 3, ValueError),                                                 # e_total below the local experts
])
def test_w4a16_rejects_bad_arguments(pos, bad, exc):
    a = _w4_args()
    a[pos] = bad
    with pytest.raises(exc):
        W4._check(*a)


def test_w4a16_has_no_cpu_path():
    with pytest.raises(ValueError, match="no CPU path"):
        W4._check(*_w4_args())
    with pytest.raises(ValueError, match="no CPU path"):
        W4.moe_w4a16(*_w4_args())


def test_proj_and_moe_have_no_cpu_path():
    from kdb200 import moe, proj, proj_f32w
    x = torch.zeros((4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        proj(x, torch.zeros((8, 64), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        proj_f32w(x, torch.zeros((8, 128), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        moe.route(x, torch.zeros((8, 64)), None, 2)


def test_moe_helpers_check_before_launch():
    from kdb200 import moe
    x = torch.zeros((4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        moe.router_approx(x, torch.zeros((8, 128), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        moe.route_fast(x, torch.zeros((8, 64)), None, torch.zeros((8, 128), dtype=torch.bfloat16), torch.zeros(8), 2)
    with pytest.raises(ValueError, match="CUDA"):
        moe.plan(torch.zeros((4, 2), dtype=torch.int32), torch.zeros((4, 2)), 8)


def test_moe_stage_entry_points_check_before_launch():
    from kdb200 import moe
    a = torch.zeros((6, 64), dtype=torch.bfloat16)
    idx = torch.zeros(6, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        moe.gather_rows(a, idx)
    with pytest.raises(ValueError, match="CUDA"):
        moe.expert_gate_up(a, torch.zeros((2, 256, 64), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        moe.expert_down(a, torch.zeros((2, 64, 64), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        moe.combine(a, idx, 3, 2)
    with pytest.raises(ValueError, match="CUDA"):
        moe.ep_regroup(torch.zeros((2, 3), dtype=torch.int32), a, True)
