"""GPU tests of the expert-parallel MoE path (kdb200.ep over libkdb200's stage entry points).

* the regroup kernel (kdb_moe_ep_regroup) against the restatement in tests/ep_cpu_ops.py;
* one rank (P = 1) and P = 4 ranks emulated on one GPU (dispatch / owner_compute / finish exchanged in
  process): every rank's output against the oracle layer for its tokens — ids exact, outputs within
  max-abs 2e-2 and relative Frobenius 1e-2;
* P = 2 real ranks over NCCL, when the box has two GPUs."""
from __future__ import annotations

import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from kdb200 import ep as EP
from kdb200 import moe as M
from kdb200 import workloads as W
from oracle import moe as om

import ep_cpu_ops  # noqa: E402  (tests/ is on sys.path via conftest)

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
MAX_ABS, REL_FRO = 2e-2, 1e-2


def _dev(wts):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in wts.items()}


def _check(y, ids, x, wts, k):
    ref = om.moe_ref(x.cpu(), wts, k)
    assert torch.equal(ids.cpu(), ref["ids"])
    c = om.compare(y, ref["y32"])
    assert c["nonfinite"] == 0 and c["max_abs"] <= MAX_ABS and c["rel_fro"] <= REL_FRO, c


@pytest.mark.parametrize("P,Er,H", [(3, 5, 64), (1, 4, 128), (8, 32, 256)])
def test_regroup_matches_restatement(P, Er, H):
    g = torch.Generator().manual_seed(P * 100 + Er)
    counts = torch.randint(0, 40, (P, Er), generator=g, dtype=torch.int32)
    counts[0, 0] = 0
    rows = int(counts.sum())
    x = torch.randn((rows, H), generator=g).to(torch.bfloat16)
    want, off_w, mt_w = ep_cpu_ops.ep_regroup(counts, x, True)
    got, off, mt = M.ep_regroup(counts.cuda(), x.cuda(), True)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), want) and torch.equal(off.cpu(), off_w) and torch.equal(mt.cpu(), mt_w)
    back, _, _ = M.ep_regroup(counts.cuda(), got, False)
    torch.cuda.synchronize()
    assert torch.equal(back.cpu(), x)


@pytest.mark.parametrize("cfg", [
    W.MoeConfig("ep1", 300, 512, 16, 256, 4, shared=1, shared_i=128),
    W.MoeConfig("ep1_skew", 1000, 256, 32, 128, 4, zipf_s=1.2),
])
def test_single_rank(cfg):
    x = W.moe_input(cfg.t, cfg.h, 4)
    wts = W.moe_weights(cfg, 4)
    layer = EP.ExpertParallelMoE(_dev(wts), cfg.k)
    y, w, ids = layer(x.cuda())
    torch.cuda.synchronize()
    _check(y, ids, x, wts, cfg.k)


def _emulate(layers, xs):
    """All-to-all between in-process ranks: owner o receives, from every source s in rank order, the
    rows s sent to o; results return the same way."""
    P = len(layers)
    sts = [layers[r].dispatch(xs[r]) for r in range(P)]
    sc = [st["send_counts"] for st in sts]                   # [P_owner, Er] per source
    send_off = [torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.long), c.sum(1).long().cpu()]), 0) for c in sc]
    backs = []
    for o in range(P):
        recv = torch.cat([sts[s]["send"][int(send_off[s][o]):int(send_off[s][o + 1])] for s in range(P)])
        recv_counts = torch.stack([sc[s][o] for s in range(P)])
        backs.append((layers[o].owner_compute(recv, recv_counts), recv_counts))
    outs = []
    for s in range(P):
        parts = []
        for o in range(P):
            back, rc = backs[o]
            start = int(rc[:s].sum())
            parts.append(back[start:start + int(rc[s].sum())])
        outs.append(layers[s].finish(sts[s], torch.cat(parts)))
    return outs


def test_four_ranks_emulated_on_one_gpu():
    cfg = W.MoeConfig("ep4", 256, 512, 32, 256, 4, shared=1, shared_i=128)
    wts = W.moe_weights(cfg, 5)
    gw = _dev(wts)
    layers = [EP.ExpertParallelMoE(gw, cfg.k, ranks=(4, r)) for r in range(4)]
    xs = [W.moe_input(cfg.t, cfg.h, 20 + r) for r in range(4)]
    outs = _emulate(layers, [x.cuda() for x in xs])
    torch.cuda.synchronize()
    for r in range(4):
        y, w, ids = outs[r]
        _check(y, ids, xs[r], wts, cfg.k)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, queue):
    import datetime
    for p in (str(ROOT), str(ROOT / "kernel-development_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from kdb200 import ep as EP_
    from kdb200 import workloads as W_
    from oracle import moe as om_
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        cfg = W_.MoeConfig("ep2", 512, 512, 32, 256, 8, shared=1, shared_i=128)
        wts = W_.moe_weights(cfg, 6)
        x = W_.moe_input(cfg.t, cfg.h, 30 + rank)
        layer = EP_.ExpertParallelMoE({k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in wts.items()},
                                      cfg.k)
        y, w, ids = layer(x.cuda())
        torch.cuda.synchronize()
        ref = om_.moe_ref(x, wts, cfg.k)
        c = om_.compare(y, ref["y32"])
        queue.put((rank, bool(torch.equal(ids.cpu(), ref["ids"])), c["max_abs"], c["rel_fro"], None))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        queue.put((rank, False, 1e9, 1e9, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, max_abs, rel, err in sorted(res):
        assert err is None, f"rank {rank}: {err}"
        assert ok and max_abs <= MAX_ABS and rel <= REL_FRO, (rank, ok, max_abs, rel)
