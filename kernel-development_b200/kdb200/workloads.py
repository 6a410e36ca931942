"""Seeded synthetic workloads for the projection and the MoE layer.

Shapes and value distributions of the benchmark workloads:

  projection   Y[M, N] = X[M, K] · W[N, K]ᵀ;  X ~ N(0, 1), W ~ N(0, 1/K), both rounded to bf16
               proj_2048:        M=128, K=N=2048
               proj_7168_m{M}:   K=N=7168, M in {16, 128, 1024, 4096, 16384}
  MoE layer    x ~ N(0, 1) bf16; router W ~ N(0, 1/H) fp32; expert weights ~ N(0, 1/fan_in) bf16
               moe_decode:   T=64,    H=4096, E=64,  I=1024, top-8
               moe_prefill:  T=8192,  H=7168, E=256, I=2048, top-8, one always-on shared expert (I=2048)
               moe_skewed:   T=16384, H=4096, E=128, I=1536, top-4, router bias giving Zipf(1.2)
                             expert popularity over a seeded expert permutation

Every tensor has its own torch.Generator seeded with (seed + tensor id [+ expert]), drawn in fp32 on
the requested device and then cast.  CPU and CUDA generators give different streams for the same
seed; parity tests always generate on one device and copy.  No public dataset is involved.
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass, asdict

import torch


@dataclass(frozen=True)
class ProjConfig:
    name: str
    m: int
    k: int
    n: int

    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    def bytes(self) -> float:
        return 2.0 * (self.m * self.k + self.n * self.k + self.m * self.n)


@dataclass(frozen=True)
class MoeConfig:
    name: str
    t: int          # tokens
    h: int          # hidden
    e: int          # routed experts
    i: int          # routed expert intermediate size
    k: int          # top-k
    shared: int = 0       # always-on shared experts (0 or 1)
    shared_i: int = 0     # shared expert intermediate size
    zipf_s: float = 0.0   # > 0: router bias giving Zipf(zipf_s) expert popularity

    def as_case(self) -> dict:
        d = asdict(self)
        d.pop("name")
        return d


PROJ_CONFIGS = {
    "proj_2048": ProjConfig("proj_2048", 128, 2048, 2048),
    **{f"proj_7168_m{m}": ProjConfig(f"proj_7168_m{m}", m, 7168, 7168) for m in (16, 128, 1024, 4096, 16384)},
}

MOE_CONFIGS = {
    "moe_decode": MoeConfig("moe_decode", 64, 4096, 64, 1024, 8),
    "moe_prefill": MoeConfig("moe_prefill", 8192, 7168, 256, 2048, 8, shared=1, shared_i=2048),
    "moe_skewed": MoeConfig("moe_skewed", 16384, 4096, 128, 1536, 4, zipf_s=1.2),
    # profiling stand-in for moe_prefill: same widths and rows per expert (256), 1/8 of the experts
    # and tokens, so an ncu capture holds ~3 GB on the device
    "moe_prefill_e32": MoeConfig("moe_prefill_e32", 1024, 7168, 32, 2048, 8, shared=1, shared_i=2048),
}

# tensor ids (added to the seed)
_TID_X, _TID_W, _TID_ROUTER, _TID_GU, _TID_DOWN, _TID_SGU, _TID_SDOWN, _TID_ZIPF = range(1, 9)


def _randn(shape, seed: int, device, std: float = 1.0, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


# ---------------------------------------------------------------------------------------------- projection
def proj_weight(k: int, n: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """W[n, k] bf16 ~ N(0, 1/k)."""
    return _randn((n, k), seed * 1000 + _TID_W, device, 1.0 / math.sqrt(k))


def proj_input(m: int, k: int, seed: int = 0, device="cpu", dist: str = "normal") -> torch.Tensor:
    """X[m, k] bf16 ~ N(0, 1).  dist="outliers": additionally 1 in 64 elements (seeded positions) scaled
    by 64, the heavy-tailed activation case of the reference's test lists (`dist = "outliers"`)."""
    x = _randn((m, k), seed * 1000 + _TID_X, device)
    if dist == "outliers":
        g = torch.Generator().manual_seed(seed * 1000 + _TID_X + 500)
        mask = (torch.rand((m, k), generator=g) < 1.0 / 64).to(x.device)
        x = torch.where(mask, (x.float() * 64).to(torch.bfloat16), x)
    elif dist != "normal":
        raise ValueError(f"unknown input distribution {dist!r}")
    return x


def proj_weight_f32(k: int, n: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """W[n, k] fp32 ~ N(0, 1/k): the router layer's fp32 weights."""
    return _randn((n, k), seed * 1000 + _TID_ROUTER, device, 1.0 / math.sqrt(k), torch.float32)


# ---------------------------------------------------------------------------------------------- MoE
def moe_input(t: int, h: int, seed: int = 0, device="cpu") -> torch.Tensor:
    return _randn((t, h), seed * 1000 + _TID_X, device)


@functools.lru_cache(maxsize=16)
def zipf_tau(e: int, s: float, samples: int = 20000, seed: int = 1234) -> tuple[float, float]:
    """(tau, fitted s): the bias scale tau for which argmax(z + b) with z ~ N(0, 1) iid over e experts
    and b_r = -s * tau * ln(r) (r = popularity rank 1..e) has top-1 counts following rank^-s.
    Fitted s is the least-squares slope of ln(count) on ln(rank) over ranks with a nonzero count."""
    g = torch.Generator().manual_seed(seed)
    z = torch.randn((samples, e), generator=g)
    logr = torch.log(torch.arange(1, e + 1, dtype=torch.float64))

    def fit(tau: float) -> float:
        b = (-s * tau * logr).to(torch.float32)
        top = torch.argmax(z + b, dim=1)
        cnt = torch.bincount(top, minlength=e).to(torch.float64)
        m = cnt > 0
        xs, ys = logr[m], torch.log(cnt[m])
        xs = xs - xs.mean()
        return float(-(xs * (ys - ys.mean())).sum() / (xs * xs).sum())

    lo, hi = 0.05, 5.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if fit(mid) < s:
            lo = mid
        else:
            hi = mid
    tau = 0.5 * (lo + hi)
    return tau, fit(tau)


def zipf_router_bias(e: int, s: float, seed: int = 0) -> torch.Tensor:
    """fp32 [e] router-logit bias: expert perm[r-1] gets -s * tau * ln(r) (seeded permutation)."""
    tau, _ = zipf_tau(e, s)
    g = torch.Generator().manual_seed(seed * 1000 + _TID_ZIPF)
    perm = torch.randperm(e, generator=g)
    ranks = torch.empty(e, dtype=torch.float64)
    ranks[perm] = torch.arange(1, e + 1, dtype=torch.float64)
    return (-s * tau * torch.log(ranks)).to(torch.float32)


def moe_weights(cfg: MoeConfig, seed: int = 0, device="cpu", experts: range | None = None) -> dict:
    """Layer weights.  w_gate_up[e] = [gate rows (I); up rows (I)] x H, w_down[e] = H x I.

    Keys: router fp32[E, H], router_bias fp32[E] or None, w_gate_up bf16[E, 2I, H],
    w_down bf16[E, H, I], shared_gate_up bf16[S, 2Is, H] or None, shared_down bf16[S, H, Is] or None.
    Expert tensors are drawn expert by expert (each from its own seed) so that no fp32 copy of a
    whole stack is ever held; `experts` restricts them to a range (an expert-parallel rank's slice,
    equal to that slice of the full layer)."""
    E, H, I = cfg.e, cfg.h, cfg.i
    ex = range(E) if experts is None else experts
    out = {
        "router": _randn((E, H), seed * 1000 + _TID_ROUTER, device, 1.0 / math.sqrt(H), torch.float32),
        "router_bias": zipf_router_bias(E, cfg.zipf_s, seed).to(device) if cfg.zipf_s > 0 else None,
    }
    gu = torch.empty((len(ex), 2 * I, H), dtype=torch.bfloat16, device=device)
    dn = torch.empty((len(ex), H, I), dtype=torch.bfloat16, device=device)
    for j, e in enumerate(ex):
        gu[j] = _randn((2 * I, H), (seed * 1000 + _TID_GU) * 4096 + e, device, 1.0 / math.sqrt(H))
        dn[j] = _randn((H, I), (seed * 1000 + _TID_DOWN) * 4096 + e, device, 1.0 / math.sqrt(I))
    out["w_gate_up"], out["w_down"] = gu, dn
    if cfg.shared:
        Is = cfg.shared_i
        out["shared_gate_up"] = torch.stack([
            _randn((2 * Is, H), (seed * 1000 + _TID_SGU) * 4096 + s, device, 1.0 / math.sqrt(H))
            for s in range(cfg.shared)])
        out["shared_down"] = torch.stack([
            _randn((H, Is), (seed * 1000 + _TID_SDOWN) * 4096 + s, device, 1.0 / math.sqrt(Is))
            for s in range(cfg.shared)])
    else:
        out["shared_gate_up"] = None
        out["shared_down"] = None
    return out


def moe_flops(cfg: MoeConfig) -> float:
    """Algorithmic FLOPs of one layer call: router GEMV, routed gate_up + down, shared expert."""
    routed = cfg.t * cfg.k * (4.0 * cfg.h * cfg.i + 2.0 * cfg.i * cfg.h)
    shared = cfg.shared * cfg.t * 6.0 * cfg.h * cfg.shared_i
    router = 2.0 * cfg.t * cfg.h * cfg.e
    return routed + shared + router


def moe_bytes(cfg: MoeConfig, distinct_experts: int) -> float:
    """Algorithmic HBM bytes: weights of the experts the routing touches, shared expert, router,
    x in and y out, routing ids/weights out (intermediates and permuted copies excluded)."""
    w = distinct_experts * 3.0 * cfg.h * cfg.i * 2
    ws = cfg.shared * 3.0 * cfg.h * cfg.shared_i * 2
    return w + ws + 4.0 * cfg.h * cfg.e + 2.0 * (2.0 * cfg.t * cfg.h) + 8.0 * cfg.t * cfg.k


# ------------------------------------------------------------------------------------ NVFP4 w4a16 MoE
# NVFP4 weights: E2M1 codes (two per byte, element 2j in the low nibble), one E4M3 scale per 16 consecutive
# elements of a row, one fp32 global scale per expert tensor; value = e2m1(code) * e4m3(scale) * global.
# e2m1(code) * e4m3(scale) has at most 6 significant bits, so it is exact in bf16: a kernel may dequantise
# to bf16 without rounding and apply the global scale to the fp32 accumulator.
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


@dataclass(frozen=True)
class W4A16Config:
    """One expert-parallel rank of an NVFP4 MoE layer: `local` experts of `e_total` live here (ids
    0..local-1), every token carries k routes over all e_total experts and only the local ones are
    computed (the reference's ep8 slice, src/kdev/adapters/okc_problems/muse_moe_w4a16.toml:136)."""
    name: str
    t: int
    h: int
    i: int
    local: int
    e_total: int
    k: int
    skew: bool = False


W4A16_CONFIGS = {
    "w4a16_bs1": W4A16Config("w4a16_bs1", 1, 4096, 4096, 32, 256, 8),
    "w4a16_bs16": W4A16Config("w4a16_bs16", 16, 4096, 4096, 32, 256, 8),
    "w4a16_bs256": W4A16Config("w4a16_bs256", 256, 4096, 4096, 32, 256, 8),
    "w4a16_bs32_skewed": W4A16Config("w4a16_bs32_skewed", 32, 4096, 4096, 32, 256, 8, skew=True),
}


# Decision boundaries between consecutive E2M1 magnitudes (midpoints of E2M1_VALUES), each with the side a
# value exactly on it goes to: the even code of the two (mantissa 0), i.e. down at 0.25, 1.25, 2.5 and 5,
# up at 0.75, 1.75 and 3.5.
_E2M1_BOUNDS = ((0.25, False), (0.75, True), (1.25, False), (1.75, True), (2.5, False), (3.5, True), (5.0, False))


def e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code (4 bits: sign, 2 exponent, 1 mantissa; ties to the even mantissa) of fp32 v,
    saturating at +-6.  Returns uint8 codes 0..15.  The magnitude code is the number of decision
    boundaries the magnitude passes."""
    mag = v.abs().clamp(max=6.0)
    idx = torch.zeros(v.shape, dtype=torch.uint8, device=v.device)
    for bound, tie_up in _E2M1_BOUNDS:
        idx += (mag >= bound) if tie_up else (mag > bound)
    idx |= ((v < 0) & (idx > 0)).to(torch.uint8) << 3
    return idx


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    """fp32 values of uint8 E2M1 codes 0..15."""
    grid = torch.tensor(E2M1_VALUES + tuple(-x for x in E2M1_VALUES), dtype=torch.float32)
    return grid[codes.long()]


def nvfp4_quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 w [rows, cols] (cols % 16 == 0) -> (codes uint8 [rows, cols/2], scales float8_e4m3fn
    [rows, cols/16], global fp32 scalar): per-16 amax / 6 scaled into E4M3's range by the global scale."""
    rows, cols = w.shape
    blocks = w.reshape(rows, cols // 16, 16)
    amax = blocks.abs().amax(-1)
    g = float(amax.max()) / (6.0 * 448.0) if float(amax.max()) > 0 else 1.0
    scale = (amax / 6.0 / g).to(torch.float8_e4m3fn)
    s = scale.float().clamp(min=2.0 ** -9)
    codes = e2m1_encode(blocks / (s.unsqueeze(-1) * g)).reshape(rows, cols)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), scale.contiguous(), torch.tensor(g, dtype=torch.float32)


def nvfp4_dequantize(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """e2m1(code) * e4m3(scale) as fp32 [rows, cols] (exactly representable in bf16); the global scale
    is not applied."""
    rows = codes.shape[0]
    lo = e2m1_decode(codes & 0xF)
    hi = e2m1_decode(codes >> 4)
    vals = torch.stack([lo, hi], dim=-1).reshape(rows, -1)
    return (vals.reshape(rows, -1, 16) * scales.float().unsqueeze(-1)).reshape(rows, -1)


def w4a16_weights(cfg: W4A16Config, seed: int = 0, experts: list[int] | None = None) -> dict:
    """NVFP4 weights of the local experts (CPU): w13 [L, 2I, H/2] uint8 (rows 0..I-1 gate, I..2I-1 up),
    w13_scale [L, 2I, H/16] e4m3, w13_gscale [L] fp32, w2 [L, H, I/2], w2_scale [L, H, I/16], w2_gscale [L],
    pw1 [H] fp32 (the per-feature output weight, shared by the rank's experts).
    `experts` restricts (and orders) the experts drawn; each is the same as in the full set."""
    H, I = cfg.h, cfg.i
    out = {k: [] for k in ("w13", "w13_scale", "w13_gscale", "w2", "w2_scale", "w2_gscale")}
    for e in (range(cfg.local) if experts is None else experts):
        w13 = _randn((2 * I, H), (seed * 1000 + _TID_GU) * 4096 + e, "cpu", 1.0 / math.sqrt(H), torch.float32)
        w2 = _randn((H, I), (seed * 1000 + _TID_DOWN) * 4096 + e, "cpu", 1.0 / math.sqrt(I), torch.float32)
        for name, w in (("w13", w13), ("w2", w2)):
            c, s, g = nvfp4_quantize(w)
            out[name].append(c)
            out[name + "_scale"].append(s)
            out[name + "_gscale"].append(g)
    res = {k: torch.stack(v) for k, v in out.items()}
    # the engines' per-feature output weight pw1 [H] (sc_h.cu:51): seeded, around 1
    res["pw1"] = 1.0 + 0.25 * _randn((H,), seed * 1000 + _TID_ZIPF + 100, "cpu", 1.0, torch.float32)
    return res


def w4a16_routing(cfg: W4A16Config, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """(topk_ids int32 [T, k] over e_total experts, topk_w fp32 [T, k] renormalised): distinct experts per
    token drawn with extra weight on the local ones (this rank is the busiest, as in the reference's
    rank='busiest' routing); skew concentrates the local routes on a few experts."""
    g = torch.Generator().manual_seed(seed * 1000 + _TID_ROUTER)
    pref = torch.ones(cfg.e_total)
    pref[: cfg.local] = 4.0
    if cfg.skew:
        pref[: cfg.local] = 4.0 * torch.pow(torch.arange(1, cfg.local + 1, dtype=torch.float32), -1.2) * 4
    ids = torch.stack([torch.multinomial(pref, cfg.k, replacement=False, generator=g) for _ in range(cfg.t)])
    logits = torch.randn((cfg.t, cfg.k), generator=g)
    w = torch.softmax(logits, dim=-1)
    return ids.to(torch.int32), w.to(torch.float32)


# ------------------------------------------------------------------------------------------------ attention
# The scored shapes of the reference's muse_attention_decode problem (okc_problems/muse_attention_decode.toml
# [[shapes]]: case and seed), named attn_<id> with "/" -> "_".
ATTN_CONFIGS = {
    "attn_d1_sliding": (dict(batch=1, ctx=80000, heads="tp8", layer="sliding", dist="soft"), 601),
    "attn_d1_full": (dict(batch=1, ctx=80000, heads="tp8", layer="full", dist="coherent"), 602),
    "attn_d16_sliding": (dict(batch=16, ctx=80000, heads="tp8", layer="sliding", spread="agentic", dist="soft"), 603),
    "attn_d16_full": (dict(batch=16, ctx=80000, heads="tp8", layer="full", spread="agentic", dist="coherent"), 604),
    "attn_d32_sliding": (dict(batch=32, ctx=80000, heads="tp8", layer="sliding", spread="agentic", dist="soft"), 605),
    "attn_d32_full": (dict(batch=32, ctx=80000, heads="tp8", layer="full", spread="agentic", dist="coherent"), 606),
    "attn_v1_sliding": (dict(batch=1, ctx=80000, heads="tp8", layer="sliding", q_len=8, dist="soft"), 607),
    "attn_v1_full": (dict(batch=1, ctx=80000, heads="tp8", layer="full", q_len=8, dist="coherent"), 608),
    "attn_v16_sliding": (dict(batch=16, ctx=80000, heads="tp8", layer="sliding", q_len=8, spread="agentic",
                              dist="soft"), 609),
    "attn_v16_full": (dict(batch=16, ctx=80000, heads="tp8", layer="full", q_len=8, spread="agentic",
                           dist="coherent"), 610),
    "attn_v32_sliding": (dict(batch=32, ctx=80000, heads="tp8", layer="sliding", q_len=8, spread="agentic",
                              dist="soft"), 611),
    "attn_v32_full": (dict(batch=32, ctx=80000, heads="tp8", layer="full", q_len=8, spread="agentic",
                           dist="coherent"), 612),
}


def attn_keys(data: dict, window: int) -> int:
    """Cached keys one call reads, summed over sequences and KV heads (each 256 B: K and V, one byte each)."""
    T = data["q"].shape[1]
    Hkv = data["k_cache"].shape[1]
    total = 0
    for L in data["seq_lens"].tolist():
        total += min(int(L), window + T - 1) if window > 0 else int(L)
    return total * Hkv
