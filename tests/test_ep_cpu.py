"""Expert-parallel host logic over a world-size-2 gloo group on the CPU.

kdb200.ep.ExpertParallelMoE runs with its device stages replaced by the CPU stand-in of
tests/ep_cpu_ops.py (oracle routing, torch experts): owner-major dispatch, the count and row
all-to-alls, the regroup order and the weighted combine must reproduce, on every rank, the
single-process oracle layer for that rank's tokens (ids exact, outputs within the layer tolerance)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_args, queue, micro_batches=None):
    import datetime
    for p in (str(ROOT), str(ROOT / "kernel-development_b200"), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    import ep_cpu_ops
    from kdb200 import ep as EP
    from kdb200 import workloads as W
    from oracle import moe as om
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        cfg = W.MoeConfig(*cfg_args)
        wts = W.moe_weights(cfg, seed=3)                  # same full layer on every rank
        x = W.moe_input(cfg.t, cfg.h, seed=10 + rank)     # each rank its own tokens
        layer = EP.ExpertParallelMoE(wts, cfg.k, ops=ep_cpu_ops)
        y, w, ids = layer(x, micro_batches=micro_batches)
        ref = om.moe_ref(x, wts, cfg.k)
        ok_ids = bool(torch.equal(ids, ref["ids"]))
        c = om.compare(y, ref["y32"])
        queue.put((rank, ok_ids, c["max_abs"], c["rel_fro"], None))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        queue.put((rank, False, 1e9, 1e9, repr(e)))


@pytest.mark.parametrize("cfg_args,micro_batches", [
    (("ep_small", 48, 64, 8, 128, 2), None),
    (("ep_shared_skew", 40, 64, 16, 128, 4, 1, 128, 1.2), None),
    # three micro-batches: asynchronous exchanges of one slice overlap another slice's expert compute
    (("ep_micro", 50, 64, 8, 128, 2, 1, 128), 3),
])
def test_expert_parallel_host_logic_gloo(cfg_args, micro_batches):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, cfg_args, q, micro_batches)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_ids, max_abs, rel, err in sorted(results):
        assert err is None, f"rank {rank}: {err}"
        assert ok_ids, f"rank {rank}: routing ids differ"
        assert max_abs <= 2e-2 and rel <= 1e-2, (rank, max_abs, rel)


def _fault_worker(rank, world, port, mode, queue):
    """Rank 1 fails between layer calls (raises and exits, or stays alive without joining the exchange);
    rank 0's next call must end with an error from its collective within the group timeout, not hang."""
    import datetime
    import time
    for p in (str(ROOT), str(ROOT / "kernel-development_b200"), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    import ep_cpu_ops
    from kdb200 import ep as EP
    from kdb200 import workloads as W
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    cfg = W.MoeConfig("fault", 24, 64, 8, 128, 2)
    layer = EP.ExpertParallelMoE(W.moe_weights(cfg, seed=3), cfg.k, ops=ep_cpu_ops)
    x = W.moe_input(cfg.t, cfg.h, seed=10 + rank)
    layer(x)                                              # one good call on both ranks
    if rank == 1:
        if mode == "stall":
            time.sleep(12)                                # alive, but never joins the next exchange
        _report_and_exit(queue, (rank, "left", 0.0))     # leaves without tearing the group down
    t0 = time.time()
    try:
        layer(x)
        res = (rank, "no error", time.time() - t0)
    except Exception as e:  # noqa: BLE001 - the expected outcome, reported to the parent
        res = (rank, type(e).__name__, time.time() - t0)
    _report_and_exit(queue, res)


def _report_and_exit(queue, item):
    queue.put(item)
    queue.close()
    queue.join_thread()                                   # flush before the hard exit
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_expert_parallel_peer_failure_is_reported_not_hung(mode):
    """Failure detection on the host (no device fault): a peer that exits between calls breaks the next
    exchange at once (connection closed); one that stays away ends it at the group's 5 s timeout."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert results[1][0] == "left"
    what, dt = results[0]
    assert what != "no error", "the surviving rank's exchange returned without its peer"
    assert dt < 30.0, f"the surviving rank took {dt:.1f} s to notice"
    if mode == "stall":
        assert dt >= 4.0, f"the exchange gave up after {dt:.1f} s, before the group timeout"
