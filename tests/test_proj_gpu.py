"""GPU parity tests of the bf16 projection (libkdb200 kdb_proj_bf16) against the fp32 oracle.

Tolerance (written here, shared with the oracle's check): max-abs <= 2e-2 * max(1, rms(Y_ref)) and relative
Frobenius <= 1e-2 against x.float() @ w.float().T; the bf16 rounding of Y alone gives ~1.7e-3.  The benchmark
distributions have rms(Y_ref) ~ 1, so the max-abs bound there is 2e-2."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from kdb200 import _lib, proj, proj_into
from kdb200 import workloads as W
from oracle import proj as op

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
MAX_ABS = 2e-2
REL_FRO = 1e-2


def _pair(m, k, n, seed=0):
    x = W.proj_input(m, k, seed)
    w = W.proj_weight(k, n, seed)
    return x, w, x.cuda(), w.cuda()


def _assert_close(y, ref):
    c = op.compare(y, ref)
    assert c["nonfinite"] == 0, c
    assert c["max_abs"] <= MAX_ABS * max(1.0, float(ref.float().pow(2).mean().sqrt())) and c["rel_fro"] <= REL_FRO, c


@pytest.mark.parametrize("m,k,n", [
    (128, 2048, 2048),     # projection config of the CPU-runnable case
    (1, 64, 256), (16, 7168, 512), (200, 300 - 4, 300), (129, 136, 257), (257, 512, 1000),
    (64, 8, 64), (512, 1024, 768), (1000, 520, 64),
])
def test_proj_matches_oracle(m, k, n):
    x, w, gx, gw = _pair(m, k, n, seed=m + n)
    y = proj(gx, gw)
    torch.cuda.synchronize()
    _assert_close(y, op.proj_ref(x, w))


@pytest.mark.parametrize("tile_n,cta_pair", [(64, 0), (128, 0), (192, 0), (224, 0), (256, 0),
                                             (192, 1), (224, 1), (256, 1)])
def test_every_tile_shape(tile_n, cta_pair):
    x, w, gx, gw = _pair(300, 256, 520, seed=tile_n + cta_pair)
    y = torch.empty((300, 520), dtype=torch.bfloat16, device="cuda")
    proj_into(gx, gw, y, tile_n=tile_n, cta_pair=cta_pair)
    torch.cuda.synchronize()
    _assert_close(y, op.proj_ref(x, w))


@pytest.mark.parametrize("m,k,n", [(128, 64, 256), (1000, 520, 700), (4096, 7168, 7168)])
def test_cta_pair_tiles_match_single_cta(m, k, n):
    """256-row tiles on 2-CTA clusters give the same result as 128-row tiles (same K order per element)."""
    gx = W.proj_input(m, k, 7, device="cuda")
    gw = W.proj_weight(k, n, 7, device="cuda")
    y1 = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    y2 = torch.empty_like(y1)
    proj_into(gx, gw, y1, tile_n=256, cta_pair=0)
    proj_into(gx, gw, y2, tile_n=256, cta_pair=1)
    torch.cuda.synchronize()
    rows = torch.arange(0, m, max(1, m // 64))
    _assert_close(y2[rows], gx[rows].cpu().float() @ gw.cpu().float().T)
    assert float((y1.float() - y2.float()).abs().max()) <= 2e-2


@pytest.mark.parametrize("m,k,n", [(1, 7168, 7168), (16, 7168, 7168), (128, 7168, 7168), (128, 2048, 2048),
                                   (37, 520, 1000), (100, 4096, 300), (5, 256, 333), (33, 64, 130)])
def test_small_m_split_k(m, k, n):
    """Weight-streaming shapes (M <= 128): swapped operands with K split over the CTAs of a cluster, whose
    fp32 partials are summed in slice order through distributed shared memory in the same launch;
    deterministic (same result twice) and within tolerance of the oracle.  Odd N exercises the scalar
    stores, K = 64 a single slice."""
    x, w, gx, gw = _pair(m, k, n, seed=m * 3 + n)
    y1 = proj(gx, gw)
    y2 = proj(gx, gw)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    _assert_close(y1, op.proj_ref(x, w))


def test_small_m_without_workspace():
    """The C entry point without a workspace runs the same single-launch path (no workspace is needed)."""
    import ctypes
    x, w, gx, gw = _pair(16, 7168, 2048, seed=3)
    y = torch.empty((16, 2048), dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().kdb_proj_bf16(gx.data_ptr(), gw.data_ptr(), y.data_ptr(), 16, 2048, 7168, 2048,
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    _assert_close(y, op.proj_ref(x, w))


def test_output_into_column_slice():
    """Column-parallel layout: write into a slice of a wider Y (row stride ldy > n)."""
    x, w, gx, gw = _pair(64, 128, 96, seed=5)
    big = torch.full((64, 256), 7.0, dtype=torch.bfloat16, device="cuda")
    proj_into(gx, gw, big[:, 64:160])
    torch.cuda.synchronize()
    _assert_close(big[:, 64:160], op.proj_ref(x, w))
    assert bool((big[:, :64] == 7).all()) and bool((big[:, 160:] == 7).all())


def test_k_zero_writes_zeros():
    gx = torch.empty((4, 0), dtype=torch.bfloat16, device="cuda")
    gw = torch.empty((8, 0), dtype=torch.bfloat16, device="cuda")
    y = proj(gx, gw)
    torch.cuda.synchronize()
    assert bool((y == 0).all())


def test_bad_arguments_raise():
    gx = torch.zeros((4, 12), dtype=torch.bfloat16, device="cuda")
    gw = torch.zeros((8, 12), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.KdbError):
        proj(gx, gw)                       # K % 8 != 0
    with pytest.raises(TypeError):
        proj(gx.float(), gw)                 # not bf16


def test_golden_fixtures():
    for name in ("proj_small", "proj_ragged"):
        f = np.load(GOLDEN / f"{name}.npz")
        x = torch.from_numpy(f["x_bits"].view(np.int16)).view(torch.bfloat16)
        w = torch.from_numpy(f["w_bits"].view(np.int16)).view(torch.bfloat16)
        y = proj(x.cuda(), w.cuda())
        torch.cuda.synchronize()
        _assert_close(y, torch.from_numpy(f["y32"]))


def test_graph_replay_bitwise_equal_to_eager():
    """kdev replays the op inside a CUDA graph with fresh inputs copied into the captured buffers."""
    x, w, gx, gw = _pair(256, 512, 768, seed=9)
    eager = proj(gx, gw).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        proj(gx, gw)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = proj(gx, gw)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    x2 = W.proj_input(256, 512, 99)
    gx.copy_(x2.cuda())
    g.replay()
    torch.cuda.synchronize()
    _assert_close(out, op.proj_ref(x2, w))


@pytest.mark.parametrize("m", [1024, 4096, 16384])
def test_full_size_sampled_rows(m):
    """K = N = 7168 sweep sizes M = 1024, 4096 (the headline configuration) and 16384: rows sampled
    across the whole output (tile edges and random rows) are checked against the oracle; row
    independence makes the sample representative."""
    k, n = 7168, 7168
    gx = W.proj_input(m, k, 3, device="cuda")
    gw = W.proj_weight(k, n, 3, device="cuda")
    y = proj(gx, gw)
    torch.cuda.synchronize()
    edges = [0, 1, 127, 128, 255, 256, m // 2 - 1, m // 2, m - 2, m - 1]
    rand = torch.randperm(m, generator=torch.Generator().manual_seed(m))[:22].tolist()
    rows = torch.tensor(sorted(set(edges + rand)))
    ref = gx[rows].cpu().float() @ gw.cpu().float().T
    _assert_close(y[rows], ref)


def test_deterministic_and_row_independent():
    """Same input twice -> bitwise equal; permuting X's rows permutes Y's rows bitwise."""
    gx = W.proj_input(384, 1024, 4, device="cuda")
    gw = W.proj_weight(1024, 512, 4, device="cuda")
    y1 = proj(gx, gw)
    y2 = proj(gx, gw)
    perm = torch.randperm(384, generator=torch.Generator().manual_seed(0)).cuda()
    y3 = proj(gx[perm].contiguous(), gw)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(y3, y1[perm])


# ------------------------------------------------------------------------- fp32 weights (router layer)
# Tolerance (the oracle's router-layer bound): relative Frobenius <= 1e-4 and max-abs <= 1e-3 against the
# fp64-accumulated product with the fp32 weights; probe rows exact to 0.1% (muse_bf16_proj.toml:376).
@pytest.mark.parametrize("m,k,n,dist", [
    (1, 7168, 256, "normal"), (8, 7168, 256, "normal"), (9, 7168, 256, "outliers"), (32, 7168, 256, "normal"),
    (33, 7168, 256, "normal"), (128, 7168, 256, "normal"), (129, 7168, 256, "normal"), (300, 7168, 256, "normal"),
    (1000, 512, 100, "outliers"), (24, 640, 130, "normal"),
])
def test_f32w_matches_oracle(m, k, n, dist):
    from kdb200 import proj_f32w, split_f32
    x = W.proj_input(m, k, m + 3, dist=dist)
    w = W.proj_weight_f32(k, n, n + 1)
    gw = w.cuda()
    split = split_f32(gw)
    assert torch.equal(gw.cpu(), w)   # the caller's weights are untouched
    y = proj_f32w(x.cuda(), split)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    ok, msg = op.check_f32w(y.cpu(), op.proj_ref_f32w(x, w))
    assert ok, msg
    # a bf16 rounding of the weights would not pass the router bound: the hi+mid pair is doing its job
    rough = op.proj_ref_f32w(x, w.to(torch.bfloat16).float())
    assert not op.check_f32w(rough, op.proj_ref_f32w(x, w))[0]


@pytest.mark.parametrize("m", [1, 16, 200])
def test_f32w_probe_rows_exact(m):
    """One nonzero power-of-two input per row returns that weight column scaled, to 0.1% per element."""
    from kdb200 import proj_f32w, split_f32
    k, n = 7168, 256
    w = W.proj_weight_f32(k, n, 11)
    g = torch.Generator().manual_seed(m)
    cols = torch.randint(0, k, (m,), generator=g)
    pw = torch.randint(-6, 7, (m,), generator=g).float()
    x = torch.zeros((m, k), dtype=torch.float32)
    x[torch.arange(m), cols] = torch.pow(2.0, pw)
    y = proj_f32w(x.to(torch.bfloat16).cuda(), split_f32(w.cuda())).cpu()
    torch.cuda.synchronize()
    want = w[:, cols].T * torch.pow(2.0, pw)[:, None]
    rel = ((y - want).abs() / want.abs().clamp_min(1e-30)).max().item()
    assert rel <= op.PROBE_REL_TOL, rel


def test_f32w_through_submission_and_graph():
    """The submission's prepare/kernel_fn route the fp32 router layer to kdb_proj_f32w; graph replay equals eager."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "b200_bf16_proj_sub", Path(__file__).resolve().parent.parent / "kernel-development_b200" / "submissions" /
        "b200_bf16_proj.py")
    sub = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sub)
    w = W.proj_weight_f32(7168, 256, 5)
    state = sub.prepare({"router": w.cuda()})
    x = W.proj_input(16, 7168, 2, device="cuda")
    data = {"x": x, "config": {"m": 16, "layer": "router"}}
    y = sub.kernel_fn(data, state)
    torch.cuda.synchronize()
    assert op.check_f32w(y.cpu(), op.proj_ref_f32w(x, w))[0]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sub.kernel_fn(data, state)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = sub.kernel_fn(data, state)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y)


def test_f32w_rejects_bad_shapes():
    from kdb200 import _lib as L
    from kdb200 import proj_f32w, split_f32
    with pytest.raises(ValueError):
        proj_f32w(torch.zeros((4, 64), dtype=torch.bfloat16, device="cuda"),
                  torch.zeros((8, 64), dtype=torch.bfloat16, device="cuda"))     # w_split not [n, 2k]
    with pytest.raises(L.KdbError):                                               # k % 64 != 0
        proj_f32w(torch.zeros((4, 72), dtype=torch.bfloat16, device="cuda"),
                  split_f32(torch.zeros((8, 72), dtype=torch.float32, device="cuda")))
