"""Expert-parallel fused MoE layer over P ranks (one process per GPU, torch.distributed NCCL).

Rank r owns experts [r*Er, (r+1)*Er) with Er = E / P and its own batch of tokens; the router and the
shared expert are replicated.  One layer call on rank r:

  1. route its tokens (bit-exact ids and weights: the single-GPU router)           kdb_moe_route_fast
  2. plan: slots grouped by expert, hence by owner rank                            kdb_moe_plan
  3. gather the token rows in that order                                           kdb_moe_gather_rows
  4. all-to-all of the per-(owner, expert) counts, then of the rows (NCCL; the row split sizes are
     read back to the host once per call, so this path is eager, not graph-captured)
  5. owner: regroup source-major blocks to expert-major                             kdb_moe_ep_regroup
  6. owner: grouped gate_up (SwiGLU) and down over its Er experts, unscaled         kdb_moe_expert_*
  7. owner: regroup back to source-major, all-to-all the rows home
  8. combine: y[t] = sum_j w[t, j] * row(t, j) (+ shared expert on local tokens)   kdb_moe_combine

The all-to-alls are issued asynchronously (NCCL runs them on its own stream) and the shared expert runs
while the dispatched rows are in flight, on all but `comm_sms` SMs (kdb_set_sm_budget): the persistent
GEMMs would otherwise hold every SM and NCCL's kernels would wait for them.  A call can also be split into
micro-batches so that one slice's exchange overlaps another slice's expert GEMMs; measured on 8 B200s that
was not faster, so it is off by default.

The reference simulates a single expert-parallel rank and computes only its local routes
(src/kdev/adapters/okc_problems/muse_moe_w4a16.toml:31,136); this is the real exchange.
"""
from __future__ import annotations

import contextlib
from typing import Optional

import torch
import torch.distributed as dist

from . import moe as M


class ExpertParallelMoE:
    """One rank's part of an expert-parallel MoE layer.

    `weights` is the full layer (router fp32 [E, H], w_gate_up [E, 2I, H], w_down [E, H, I], optional
    router_bias and shared expert) or only this rank's expert slice when `local_experts=True`
    (w_gate_up/w_down then hold Er experts).  Tensors must be on this rank's GPU.
    """

    def __init__(self, weights: dict, k: int, group: Optional[dist.ProcessGroup] = None,
                 local_experts: bool = False, ranks: Optional[tuple[int, int]] = None, ops=None):
        """`ranks` = (P, rank) places this instance in a P-rank layout without a process group (several
        instances in one process exchange rows through dispatch / owner_compute / finish).  `ops` is
        the module of device stages (default kdb200.moe, the libkdb200 kernels); a test harness may pass
        a stand-in with the same functions to exercise this host logic elsewhere."""
        self.group = group
        self.ops = M if ops is None else ops
        if ranks is not None:
            self.P, self.rank = int(ranks[0]), int(ranks[1])
        else:
            self.P = dist.get_world_size(group) if dist.is_initialized() else 1
            self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        router = weights["router"].contiguous()
        self.E = router.shape[0]
        if self.E % self.P:
            raise ValueError(f"{self.E} experts do not split over {self.P} ranks")
        self.Er = self.E // self.P
        self.k = int(k)
        gu, dn = weights["w_gate_up"], weights["w_down"]
        if not local_experts:
            sl = slice(self.rank * self.Er, (self.rank + 1) * self.Er)
            gu, dn = gu[sl], dn[sl]
        if gu.shape[0] != self.Er:
            raise ValueError(f"expected {self.Er} local experts, got {gu.shape[0]}")
        self.router = router
        bias = weights.get("router_bias")
        self.router_bias = None if bias is None else bias.to(router.device).contiguous()
        ops = self.ops
        self.split, self.norms = (ops.prepare_router(router) if router.shape[1] % 64 == 0 else (None, None))
        self.w_gate_up_packed = ops.pack_gate_up(gu.contiguous())
        self.w_down = dn.contiguous()
        sgu = weights.get("shared_gate_up")
        self.shared_gate_up_packed = None if sgu is None else ops.pack_gate_up(sgu.contiguous())
        self.shared_down = None if sgu is None else weights["shared_down"].contiguous()

    # -------------------------------------------------------------------------------------------------
    def _route(self, x: torch.Tensor):
        if self.split is not None:
            return self.ops.route_fast(x, self.router, self.router_bias, self.split, self.norms, self.k)
        _, w, ids = self.ops.route(x, self.router, self.router_bias, self.k)
        return w, ids

    # Phases of one call (forward composes them around the two all-to-alls; tests on one GPU emulate
    # the exchange between several instances).
    def dispatch(self, x: torch.Tensor) -> dict:
        """Route this rank's tokens and lay their rows out owner-major.  Returns the call state with
        send rows [T*k, H] and send_counts int32 [P, Er] (rows for owner p's local expert e)."""
        w, ids = self._route(x)
        plan = self.ops.plan(ids, w, self.E)
        send = self.ops.gather_rows(x, plan["perm_slot"], div=self.k)
        return {"x": x, "w": w, "ids": ids, "slot_pos": plan["slot_pos"], "send": send,
                "send_counts": plan["counts"].view(self.P, self.Er)}

    def owner_compute(self, recv: torch.Tensor, recv_counts: torch.Tensor) -> torch.Tensor:
        """Owner side: rows received source-major (counts int32 [P, Er]) -> expert outputs, unscaled,
        in the same source-major order."""
        ops = self.ops
        grouped, offsets, mtile = ops.ep_regroup(recv_counts, recv, to_expert_major=True)
        hbuf = ops.expert_gate_up(grouped, self.w_gate_up_packed, offsets, mtile)
        yg = ops.expert_down(hbuf, self.w_down, offsets, mtile)
        back, _, _ = ops.ep_regroup(recv_counts, yg, to_expert_major=False)
        return back

    def shared_rows(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        """The shared expert's output rows for local tokens x (None without a shared expert)."""
        if self.shared_gate_up_packed is None:
            return None
        hs = self.ops.expert_gate_up(x, self.shared_gate_up_packed[0:1])
        return self.ops.expert_down(hs, self.shared_down[0:1])

    def finish(self, st: dict, ret: torch.Tensor, shared: Optional[torch.Tensor] = None):
        """Weighted combine of the returned rows (+ shared expert on the local tokens; computed here
        unless the caller passes its rows)."""
        x = st["x"]
        T = x.shape[0]
        if shared is None and self.shared_gate_up_packed is not None:
            shared = self.shared_rows(x)
        y = self.ops.combine(ret, st["slot_pos"], T, self.k, slot_w=st["w"], shared_rows=shared)
        return y, st["w"], st["ids"]

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        """Row all-to-all; asynchronous when P > 1 (returns the work handle to wait on, else None)."""
        if self.P == 1:
            out.copy_(inp)
            return None
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=True)

    def forward(self, x: torch.Tensor, micro_batches: Optional[int] = None, comm_sms: int = 16):
        """x bf16 [T_r, H] (this rank's tokens) -> (y bf16 [T_r, H], topk_w fp32 [T_r, k], topk_ids int32).

        micro_batches: token slices whose exchanges overlap each other's expert GEMMs (default 1).  Measured
        on 8 B200s (prefill layer, ms per call): one slice 9.70, one slice with the shared expert on 132 SMs
        beside the dispatch 9.58, two slices 10.39 / 10.45 / 9.72 with 0 / 16 / 32 SMs left to NCCL, so the
        default is one slice.  Every rank must use the same count (each slice is one round of all-to-alls).
        comm_sms: SMs the kernels that run while an exchange is in flight leave to NCCL (the persistent
        GEMMs otherwise hold every SM and NCCL's kernels wait for them); 0 = no reservation."""
        T, H = x.shape
        nb = max(1, min(int(1 if micro_batches is None else micro_batches), max(T, 1)))
        bounds = [T * i // nb for i in range(nb + 1)]
        sts = [self.dispatch(x[bounds[i]:bounds[i + 1]]) for i in range(nb)]
        # the counts of every micro-batch in one exchange, then the one host read-back of the split sizes
        send_counts = torch.stack([st["send_counts"] for st in sts])          # [nb, P, Er]
        recv_counts = torch.empty_like(send_counts)
        if self.P > 1:
            self._count_exchange(recv_counts, send_counts)
        else:
            recv_counts.copy_(send_counts)
        both = torch.stack([send_counts.sum(2), recv_counts.sum(2)]).cpu()    # [2, nb, P]
        recvs, works = [], []
        for i, st in enumerate(sts):
            send_rows, recv_rows = both[0, i].tolist(), both[1, i].tolist()
            recv = torch.empty((int(sum(recv_rows)), H), dtype=st["send"].dtype, device=x.device)
            works.append(self._exchange(recv, st["send"], recv_rows, send_rows))
            recvs.append((recv, send_rows, recv_rows))
        leave = comm_sms if self.P > 1 else 0
        with self._sm_budget(leave):
            # the shared expert needs no exchange: it runs while the first rows are in flight
            shared = [self.shared_rows(st["x"]) for st in sts]
        rets = []
        for i in range(nb):
            if works[i] is not None:
                works[i].wait()                      # the compute stream waits for this slice's rows only
            recv, send_rows, recv_rows = recvs[i]
            # with several slices another slice's exchange is in flight during this compute
            with self._sm_budget(leave if nb > 1 else 0):
                back = self.owner_compute(recv, recv_counts[i])
            ret = torch.empty(((bounds[i + 1] - bounds[i]) * self.k, H), dtype=back.dtype, device=x.device)
            rets.append((ret, self._exchange(ret, back, send_rows, recv_rows), back))
        outs = []
        for i, st in enumerate(sts):
            ret, work, _back = rets[i]                       # _back stays referenced until its send is done
            if work is not None:
                work.wait()
            outs.append(self.finish(st, ret, shared[i]))
        if nb == 1:
            return outs[0]
        return tuple(torch.cat([o[j] for o in outs]) for j in range(3))

    @contextlib.contextmanager
    def _sm_budget(self, leave: int):
        """Caps the persistent kernels' grids at (SMs - leave) for the launches inside the block."""
        if leave <= 0 or self.ops is not M:
            yield
            return
        lib = M._lib.lib()
        total = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        prev = lib.kdb_set_sm_budget(max(2, total - int(leave)))
        try:
            yield
        finally:
            lib.kdb_set_sm_budget(prev)

    def _count_exchange(self, recv_counts: torch.Tensor, send_counts: torch.Tensor) -> None:
        """recv_counts[b, s] = what rank s sent here in micro-batch b (send_counts[b, p] went to rank p)."""
        nb = send_counts.shape[0]
        snd = send_counts.transpose(0, 1).contiguous()            # [P, nb, Er]: destination-major
        rcv = torch.empty_like(snd)                               # [P, nb, Er]: source-major
        dist.all_to_all_single(rcv.view(self.P, -1), snd.view(self.P, -1), group=self.group)
        recv_counts.copy_(rcv.transpose(0, 1))

    __call__ = forward
