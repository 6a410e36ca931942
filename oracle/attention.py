"""Oracle for fp8-KV paged decode / verify attention (test infrastructure; see oracle/__init__.py).

The reference's `muse_attention_decode` problem (src/kdev/adapters/okc_problems/muse_attention_decode.toml)
has no reference.py in the reference's tree, so this module restates the computation from what the TOML and
the judge fixture pin, and names every other choice.

Pinned by the reference's files:
  * the cases: batch, ctx, q_len (1 = decode, 8 = verify), layer = sliding | full, heads = tp8 | dp, page,
    kv_scale, spread, dist (muse_attention_decode.toml [[shapes]], [[tests]], [[extra]]);
  * a sliding layer attends its 2,048-key window, a full layer the whole context, and no key is skipped
    (muse_attention_decode.toml [comply] notes);
  * the KV cache is FP8 E4M3, queries bf16 (or FP8 E4M3), and kernel_fn appends the new tokens' K/V to the
    cache (muse_attention_decode.toml [comply] precision, notes);
  * tp8 holds one KV head of dim 128 per GPU: floor_us of the full-context shapes (4.3 us for one sequence of
    80,000 tokens at the H200's 4.8 TB/s) is 256 B per cached token, K and V at one byte per element;
  * the check: relative L2 error against the reference, bound = 2.5 x the reference's own error when its
    queries are FP8 E4M3 + 0.015 (tests/fixtures/judge/judge_attention.json, records[event=test].message).
Chosen here (not pinned by the reference's files):
  * 8 query heads per KV head (tp8: 8 query / 1 KV head; dp: 64 / 8), softmax scale 1/sqrt(128);
  * page = 1 as a token-granular page table: block_table[b, j] is the cache slot of token j of sequence b;
  * a cached value is e4m3 x kv_scale (kv_scale defaults to 1);
  * the spread and dist generators of generate_input (documented there).  Their values are not the
    reference's: the fp8-query yardstick of the check comes out at 0.02-0.03 here on the shapes of the
    reference's tests t0-t7, where the fixture reports 0.053-0.092.  Parity with the reference's own problem
    is therefore unpinned; the bound formula is the reference's.

Math, per sequence b of L tokens after the append (the q_len new tokens are positions L - q_len .. L - 1),
query position p, query head h, KV head g = h // (Hq / Hkv):
  keys j in [lo, p], lo = max(0, p - window + 1) for a sliding layer (window 2048), 0 for a full layer
  s_j = (q[b, p, h] . K[b, j, g]) / sqrt(128)          fp32, K read back from the fp8 cache
  out[b, p, h] = sum_j softmax(s)_j V[b, j, g]          fp32 (bf16 on the GPU)
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

HEAD_DIM = 128
WINDOW = 2048
HEAD_LAYOUTS = {"tp8": (8, 1), "dp": (64, 8)}    # (query heads, KV heads) on one GPU
BOUND_FACTOR = 2.5
BOUND_FLOOR = 0.015
FP8_MAX = 448.0


@dataclass(frozen=True)
class AttnCase:
    batch: int
    ctx: int
    heads: str = "tp8"
    layer: str = "full"
    q_len: int = 1
    page: int = 1
    spread: str = "none"
    dist: str = "soft"
    kv_scale: float = 1.0

    @classmethod
    def from_dict(cls, case: dict) -> "AttnCase":
        keys = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in case.items() if k in keys})

    @property
    def q_heads(self) -> int:
        return HEAD_LAYOUTS[self.heads][0]

    @property
    def kv_heads(self) -> int:
        return HEAD_LAYOUTS[self.heads][1]


def seq_lens(case: AttnCase, gen: torch.Generator) -> torch.Tensor:
    """Lengths after the append, int64 [batch], each >= q_len.
    spread "none": every sequence ctx long; "mixed": uniform in [ctx / 8, ctx]; "agentic": sequence 0 at ctx,
    the others log-uniform in [ctx / 16, ctx] (a few long contexts among shorter ones)."""
    b, ctx = case.batch, case.ctx
    if case.spread in ("none", None):
        lens = torch.full((b,), ctx, dtype=torch.int64)
    elif case.spread == "mixed":
        lo = max(1, ctx // 8)
        lens = torch.randint(lo, ctx + 1, (b,), generator=gen)
    elif case.spread == "agentic":
        u = torch.rand((b,), generator=gen, dtype=torch.float64)
        lens = torch.exp(math.log(max(1, ctx // 16)) + u * (math.log(ctx) - math.log(max(1, ctx // 16)))).long()
        lens[0] = ctx
    else:
        raise ValueError(f"unknown spread {case.spread!r}")
    return lens.clamp(min=case.q_len, max=ctx)


def quantize_kv(x: torch.Tensor, kv_scale: float) -> torch.Tensor:
    """fp32/bf16 -> float8_e4m3fn of x / kv_scale, saturating at +-448."""
    return (x.float() / kv_scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def generate_input(case: AttnCase | dict, seed: int) -> dict:
    """Seeded inputs (CPU): q [B, q_len, Hq, D] bf16; k_new, v_new [B, q_len, Hkv, D] bf16; k_cache, v_cache
    [slots, Hkv, D] float8_e4m3fn holding the first L - q_len tokens of every sequence; block_table
    [B, max L] int32 (slot of each token, -1 past the end; the new tokens' slots are reserved, not written);
    seq_lens [B] int32.
    dist "soft": q, K, V ~ N(0, 1), so attention is spread over many keys; "coherent": 1 key in 64 of each
    sequence carries its KV group's mean query direction (scores a few units above the rest), so attention
    concentrates on them; "edges": the first and last key of every query's window carry it, so the window
    boundaries decide the result."""
    case = AttnCase.from_dict(case) if isinstance(case, dict) else case
    g = torch.Generator().manual_seed(int(seed))
    B, T, Hq, Hkv, D = case.batch, case.q_len, case.q_heads, case.kv_heads, HEAD_DIM
    lens = seq_lens(case, g)
    max_len = int(lens.max())
    total = int(lens.sum())
    slots = torch.randperm(total, generator=g)              # page = 1: any token may sit in any slot
    block_table = torch.full((B, max_len), -1, dtype=torch.int32)
    off = 0
    for b in range(B):
        L = int(lens[b])
        block_table[b, :L] = slots[off:off + L].to(torch.int32)
        off += L
    q = torch.randn((B, T, Hq, D), generator=g)
    k_all = torch.randn((total, Hkv, D), generator=g)       # indexed by slot
    v_all = torch.randn((total, Hkv, D), generator=g)
    if case.dist in ("coherent", "edges"):
        group = Hq // Hkv
        for b in range(B):
            L = int(lens[b])
            dirs = q[b].reshape(T, Hkv, group, D).mean(dim=(0, 2))          # [Hkv, D]: the group's mean query
            dirs = dirs / dirs.norm(dim=-1, keepdim=True) * 12.0            # scores of a few units above the rest
            if case.dist == "coherent":
                pos = torch.nonzero(torch.rand((L,), generator=g) < 1.0 / 64).flatten()
            else:
                ends = []
                for t in range(T):
                    p = L - T + t
                    ends += [max(0, p - WINDOW + 1) if case.layer == "sliding" else 0, p]
                pos = torch.tensor(sorted(set(ends)), dtype=torch.int64)
            sl = block_table[b, pos].long()
            k_all[sl] = k_all[sl] * 0.25 + dirs
    elif case.dist != "soft":
        raise ValueError(f"unknown dist {case.dist!r}")
    new_slots = torch.stack([block_table[b, int(lens[b]) - T:int(lens[b])].long() for b in range(B)])   # [B, T]
    k_new = k_all[new_slots].to(torch.bfloat16)
    v_new = v_all[new_slots].to(torch.bfloat16)
    k_cache = quantize_kv(k_all, case.kv_scale)
    v_cache = quantize_kv(v_all, case.kv_scale)
    zero = torch.zeros((), dtype=torch.float8_e4m3fn)
    k_cache[new_slots.flatten()] = zero                       # not yet appended
    v_cache[new_slots.flatten()] = zero
    return {"q": q.to(torch.bfloat16), "k_new": k_new, "v_new": v_new, "k_cache": k_cache, "v_cache": v_cache,
            "block_table": block_table, "seq_lens": lens.to(torch.int32), "kv_scale": float(case.kv_scale),
            "config": {"layer": case.layer, "heads": case.heads, "q_len": T}}


def append_kv(data: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """The caches after the new tokens' K/V are written (fp8 of value / kv_scale) into their slots."""
    kc, vc = data["k_cache"].clone(), data["v_cache"].clone()
    T = data["q"].shape[1]
    for b in range(data["q"].shape[0]):
        L = int(data["seq_lens"][b])
        sl = data["block_table"][b, L - T:L].long()
        kc[sl] = quantize_kv(data["k_new"][b], data["kv_scale"])
        vc[sl] = quantize_kv(data["v_new"][b], data["kv_scale"])
    return kc, vc


def attention_ref(data: dict, fp8_queries: bool = False, window: int | None = None) -> torch.Tensor:
    """fp32 [B, q_len, Hq, D] output after appending the new tokens (the new keys are read back from the
    fp8 cache like every other key).  fp8_queries: queries rounded to E4M3 first (the check's yardstick).
    window: keys per sliding window (default 2048; smaller values exist for tests)."""
    win = WINDOW if window is None else int(window)
    sliding = data["config"]["layer"] == "sliding"
    kc, vc = append_kv(data)
    q = data["q"].float()
    if fp8_queries:
        q = q.to(torch.float8_e4m3fn).float()
    B, T, Hq, D = q.shape
    Hkv = kc.shape[1]
    group = Hq // Hkv
    scale = 1.0 / math.sqrt(D)
    out = torch.empty((B, T, Hq, D), dtype=torch.float32)
    for b in range(B):
        L = int(data["seq_lens"][b])
        lo_all = max(0, L - T - win + 1) if sliding else 0
        sl = data["block_table"][b, lo_all:L].long()
        K = kc[sl].float() * data["kv_scale"]                        # [n, Hkv, D]
        V = vc[sl].float() * data["kv_scale"]
        pos = torch.arange(lo_all, L)
        qb = q[b].reshape(T, Hkv, group, D)
        s = torch.einsum("tgqd,ngd->tgqn", qb, K) * scale           # [T, Hkv, group, n]
        p = torch.arange(L - T, L).view(T, 1)
        keep = pos.view(1, -1) <= p
        if sliding:
            keep &= pos.view(1, -1) > p - win
        s = s.masked_fill(~keep.view(T, 1, 1, -1), float("-inf"))
        a = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("tgqn,ngd->tgqd", a, V).reshape(T, Hq, D)
    return out


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """Relative L2 error over the whole output and its worst (sequence, position, head) row."""
    o, r = out.float().reshape(-1, out.shape[-1]), ref.float().reshape(-1, ref.shape[-1])
    rel = float((o - r).norm() / r.norm().clamp_min(1e-30))
    rows = (o - r).norm(dim=1) / r.norm(dim=1).clamp_min(1e-30)
    return {"rel_l2": rel, "worst_row": float(rows.max()), "nonfinite": int((~torch.isfinite(o)).sum())}


def check(data: dict, out: torch.Tensor, window: int | None = None) -> tuple[bool, str]:
    """(ok, message) with the reference's bound: 2.5 x the fp8-query reference's own error + 0.015.
    window: keys per sliding window (default 2048; smaller values exist for tests)."""
    ref = attention_ref(data, window=window)
    yard = compare(attention_ref(data, fp8_queries=True, window=window), ref)["rel_l2"]
    bound = BOUND_FACTOR * yard + BOUND_FLOOR
    c = compare(out, ref)
    ok = c["nonfinite"] == 0 and c["rel_l2"] <= bound
    msg = (f"relative L2 error {c['rel_l2']:.3e} (worst row {c['worst_row']:.3e}) [bound {bound:.3f}: "
           f"{BOUND_FACTOR} x the reference's {yard:.3f} with FP8 E4M3 queries + {BOUND_FLOOR}]")
    return ok, msg
