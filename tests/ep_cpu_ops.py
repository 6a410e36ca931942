"""CPU stand-in for the device stages kdb200.ep drives (test helper, built on the oracle).

It implements the same functions as kdb200.moe's stage wrappers with torch on the CPU, so the
expert-parallel host logic (owner-major dispatch, split sizes, regroup order, combine) can run over a
gloo process group without a GPU.  The regroup restatement is also the reference the GPU regroup
kernel is checked against."""
from __future__ import annotations

import torch

from oracle import moe as om


def prepare_router(router):
    return None, None          # the stand-in routes through route()


def pack_gate_up(w):
    return w                   # unpacked: gate rows then up rows


def route(x, router, bias, k):
    """(logits, topk_w, topk_ids), the order of kdb200.moe.route."""
    lg, ids, w = om.route(x, router, bias, k)
    return lg, w, ids


def plan(ids, w, e):
    return om.permute(ids, e)


def gather_rows(x, index, div=1, rows=None):
    return x[index.long() // div].contiguous()


def regroup_offsets(counts: torch.Tensor):
    """(so, eo) [P, Er]: source-major and expert-major starting rows of every block (s, e)."""
    c = counts.long()
    P, Er = c.shape
    so = torch.zeros_like(c)
    eo = torch.zeros_like(c)
    run = 0
    for s in range(P):
        for e in range(Er):
            so[s, e] = run
            run += int(c[s, e])
    run = 0
    for e in range(Er):
        for s in range(P):
            eo[s, e] = run
            run += int(c[s, e])
    return so, eo


def ep_regroup(counts, rows_in, to_expert_major, rows_out=None):
    c = counts.long()
    P, Er = c.shape
    so, eo = regroup_offsets(counts)
    col = c.sum(0)
    offsets = torch.zeros(Er + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(col, 0).to(torch.int32)
    mt = (col + 511) // 512   # KDB_MOE_TOKEN_TILE
    mtile = torch.zeros(Er + 1, dtype=torch.int32)
    mtile[1:] = torch.cumsum(mt, 0).to(torch.int32)
    if rows_in is None:
        return None, offsets, mtile
    out = torch.empty_like(rows_in) if rows_out is None else rows_out
    for s in range(P):
        for e in range(Er):
            n = int(c[s, e])
            a, b = (int(so[s, e]), int(eo[s, e])) if to_expert_major else (int(eo[s, e]), int(so[s, e]))
            out[b:b + n] = rows_in[a:a + n]
    return out, offsets, mtile


def _groups(offsets, rows, n_groups):
    if offsets is None:
        return [(0, 0, rows)]
    o = offsets.tolist()
    return [(g, o[g], o[g + 1]) for g in range(n_groups)]


def expert_gate_up(a, w_packed, offsets=None, mtile_start=None):
    groups, two_i, _ = w_packed.shape
    i = two_i // 2
    out = torch.empty((a.shape[0], i), dtype=torch.bfloat16)
    for g, r0, r1 in _groups(offsets, a.shape[0], groups):
        if r1 > r0:
            gu = w_packed[g].float()
            xa = a[r0:r1].float()
            out[r0:r1] = (torch.nn.functional.silu(xa @ gu[:i].T) * (xa @ gu[i:].T)).to(torch.bfloat16)
    return out


def expert_down(a, w_down, offsets=None, mtile_start=None, row_scale=None):
    groups, h, _ = w_down.shape
    out = torch.empty((a.shape[0], h), dtype=torch.bfloat16)
    for g, r0, r1 in _groups(offsets, a.shape[0], groups):
        if r1 > r0:
            y = a[r0:r1].float() @ w_down[g].float().T
            if row_scale is not None:
                y = y * row_scale[r0:r1, None]
            out[r0:r1] = y.to(torch.bfloat16)
    return out


def combine(rows, slot_pos, t, k, slot_w=None, shared_rows=None):
    h = rows.shape[1]
    y = torch.zeros((t, h))
    sp = slot_pos.long().view(t, k)
    for j in range(k):
        r = rows[sp[:, j]].float()
        y += r * slot_w.view(t, k)[:, j:j + 1] if slot_w is not None else r
    if shared_rows is not None:
        y += shared_rows.float()
    return y.to(torch.bfloat16)
