"""Seeded synthetic workloads for the projection and the MoE layer.

Shapes and value distributions follow the benchmark configurations of this build:

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
