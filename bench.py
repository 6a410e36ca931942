#!/usr/bin/env python
"""bench.py — throughput of the B200 fused MoE layer and bf16 projection, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU, NCCL)

Default workload: moe_prefill, the MoE layer the >=55 %-of-roofline and >=6x-at-8-GPUs targets are quoted on
(T=8192 tokens, H=7168, 256 routed experts of I=2048 plus one shared expert, top-8; expert-parallel at
N > 1 with T tokens and E/N experts per GPU).  The same line nests, under "projection", the
Y[4096, 7168] = X[4096, 7168] . W[7168, 7168]^T projection (the >=70 %-of-bf16-peak target; column-parallel
over N, no collective).  Other workloads: proj_2048, proj_7168_m{16,128,1024,4096,16384}, moe_decode,
moe_skewed, moe_prefill_e32, w4a16_* (see kernel-development_b200/kdb200/workloads.py).

A step is one pass of the op over one batch already resident in HBM, replayed from a CUDA graph (the
expert-parallel layer runs eagerly).  The L2 is flushed (a 512 MiB device write, then a read of it, untimed)
before every timed step; each step is timed with CUDA events on its own stream; the time is the max over
ranks.  "e2e" repeats the measurement through the kdev-facing submission call with the inputs copied in
from pinned host memory and the outputs copied back inside each timed step.

--impl reference times the path's PyTorch fp32 formulation (the oracle) on this host's cores on a bounded
sample of the same workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "kernel-development_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

DEFAULT_WORKLOAD = "moe_prefill"
NESTED_PROJ_WORKLOAD = "proj_7168_m4096"
PROJ_METRIC = "achieved TFLOP/s of the bf16 projection (% of bf16 tensor peak in roofline.frac)"
FLUSH_BYTES = 512 << 20
PROFILES = ROOT / "profiles"


# ------------------------------------------------------------------------------------------------ utils
def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _profile_traffic(kernel_key: str, workload: str) -> float | None:
    """dram bytes per launch recorded in profiles/<kernel_key>_<workload>.txt ("traffic_bytes_per_launch: N")."""
    f = PROFILES / f"{kernel_key}_{workload}.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML every `period` s while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period: float = 0.005):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.ok = False
        self._stop = threading.Event()
        self._period = period
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        try:
            mhz = self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM)
            rs = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.samples.append((int(mhz), int(rs)))
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self._period)

    def __enter__(self):
        if self.ok:
            self._sample()
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        reasons = set()
        for _, r in self.samples:
            for name, bit in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def _flusher(dev):
    """L2 flush before a timed step: write a buffer 4x the L2, then read it back, so the L2 holds only
    clean lines of the flush buffer and the timed step pays no write-back of the flush's dirty lines
    (kdev's protocol flushes with a read for the same reason)."""
    buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        buf.fill_(1.0)
        torch.amax(buf, dim=0, out=sink)
    return flush


def _capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def timed_steps(step, steps: int, warmup: int, flush, dist: Dist, sampler: ClockSampler | None):
    """Per-step device times (ms) of `step`, each after an untimed L2 flush; bracketed by a barrier and
    a synchronize on both sides.  Returns (per-step ms list, elapsed ms of the whole timed region)."""
    for _ in range(warmup):
        flush()
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    region0, region1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        region0.record()
        for a, b in ev:
            flush()
            a.record()
            step()
            b.record()
        region1.record()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev], region0.elapsed_time(region1)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


# ------------------------------------------------------------------------------------------------ projection
def _proj_cfg(name):
    from kdb200 import workloads as W
    return W.PROJ_CONFIGS[name]


def bench_proj(args, dist: Dist) -> dict | None:
    from kdb200 import proj_into
    from kdb200 import workloads as W
    import importlib.util

    cfg = _proj_cfg(args.workload)
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    x = W.proj_input(cfg.m, cfg.k, seed=1, device=dev)
    w = W.proj_weight(cfg.k, cfg.n, seed=100 + dist.rank, device=dev)   # this rank's column shard
    y = torch.empty((cfg.m, cfg.n), dtype=torch.bfloat16, device=dev)
    flush = _flusher(dev)
    g = _capture(lambda: proj_into(x, w, y))
    sampler = ClockSampler(_physical_index(dist.local)) if dist.rank == 0 else None
    per_step, region_ms = timed_steps(g.replay, args.steps, args.warmup, flush, dist, sampler)
    ms = dist.max(sum(per_step) / len(per_step))
    flops_rank = cfg.flops()
    value = flops_rank * dist.world / (ms * 1e-3) / 1e12

    # e2e: the public kdev-facing call (submission kernel_fn) with host buffers; H2D of x and D2H of y
    # inside the timed region, every step.
    spec = importlib.util.spec_from_file_location(
        "b200_bf16_proj_sub", ROOT / "kernel-development_b200" / "submissions" / "b200_bf16_proj.py")
    sub = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sub)
    state = sub.prepare({_layer_key(cfg): w})
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((cfg.m, cfg.n), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        out = sub.kernel_fn({"x": x_dev, "config": {"m": cfg.m, "layer": _layer_key(cfg)}}, state)
        y_host.copy_(out, non_blocking=True)

    e2e_steps, _ = timed_steps(e2e_step, max(3, args.steps // 4), 2, flush, dist, None)
    e2e_ms = dist.max(statistics.mean(e2e_steps))
    e2e_value = flops_rank * dist.world / (e2e_ms * 1e-3) / 1e12
    if not torch.equal(y_host.to(dev), y):
        raise RuntimeError("e2e output differs from the device-resident run")

    if dist.rank != 0:
        return None
    peaks = _peaks()
    achieved = flops_rank / (statistics.mean(per_step) * 1e-3) / 1e12
    traffic = _profile_traffic("proj_gemm", args.workload)
    bound = "tensor" if cfg.m >= 1024 else "hbm"
    if bound == "tensor":
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops"], 4)}
    else:
        gbs = cfg.bytes() / (statistics.mean(per_step) * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(gbs / peaks["hbm_gbs"], 4)}
    roof["traffic"] = traffic
    roof["peak_source"] = f"{peaks['source']} (burst)"
    from kdb200.proj import tile_shape
    bn, pair = tile_shape(cfg.m, cfg.n)
    if cfg.m <= 128:
        roof["kernel"] = ("gemm_splitk_kernel (weights as the M operand, K split over a cluster reduced in "
                          "distributed shared memory), one launch per step")
    else:
        roof["kernel"] = (f"gemm_tn_pair_kernel<ProjSched<256,{bn}>> (256 x {bn} tiles on 2-CTA clusters)" if pair else
                          f"gemm_tn_kernel<ProjSched<128,{bn}>> (128 x {bn} tiles)") + ", one launch per step"
    line = {
        "metric": PROJ_METRIC,
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded X~N(0,1), W~N(0,1/K), bf16)",
        "config": _proj_config(cfg, dist.world, args.workload),
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": y.numel() * 2,
                "path": "submissions/b200_bf16_proj.py kernel_fn (kdev adapter API) -> kdb_proj_bf16",
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": args.steps,
        "roofline": roof,
        "clocks": sampler.summary() if sampler else None,
        "timed_region_ms": round(region_ms, 2),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_proj(cfg, args.cpu_seconds)
    return line


def _layer_key(cfg) -> str:
    return f"k{cfg.k}_n{cfg.n}"


def _physical_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local < len(parts) and parts[local].strip().isdigit():
            return int(parts[local])
    return local


# ------------------------------------------------------------------------------------------------ CPU baseline
def _cpu_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_baseline_proj(cfg, seconds: float, steps: int | None = None) -> dict:
    """Oracle fp32 projection on the host cores over a bounded row sample of the workload."""
    from kdb200 import workloads as W
    from oracle import proj as op

    cores = _cpu_threads()
    w = W.proj_weight(cfg.k, cfg.n, seed=100)
    rows = min(cfg.m, 256)
    x = W.proj_input(rows, cfg.k, seed=1)
    op.proj_ref(x, w)            # warm-up
    rates, t_end = [], time.perf_counter() + seconds
    n = 0
    while (steps is None and (time.perf_counter() < t_end or n < 3)) or (steps is not None and n < steps):
        t0 = time.perf_counter()
        op.proj_ref(x, w)
        dt = time.perf_counter() - t0
        rates.append(2.0 * rows * cfg.k * cfg.n / dt / 1e12)
        n += 1
    return {"value": round(statistics.median(rates), 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of {cfg.m} rows of X against the full W[{cfg.n}, {cfg.k}], fp32 torch matmul "
                      f"(oracle/proj.py), median of {n} runs"}


# ------------------------------------------------------------------------------------------------ MoE
MOE_LAUNCHES_PER_CALL = {
    # router pre-pass GEMM, candidates, exact top-k; plan count/scan/scatter; gather; grouped gate_up;
    # grouped down; combine; [shared expert gate_up + down]
    "base": 10, "shared": 2,
    # expert parallel: two regroups of two kernels each
    "ep": 4,
}


def _time_dominant_gate_up(state, x, cfg, flush, steps: int) -> dict:
    """The layer's dominant kernel, the grouped SwiGLU gate_up GEMM, timed alone: its inputs (the routed
    and permuted rows and the plan) are built once by the stage entry points, then each timed launch
    follows an untimed L2 flush.  Returns its mean ms and algorithmic FLOPs per launch."""
    from kdb200 import moe as M
    w, ids = M.route_fast(x, state["router"], state["router_bias"], state["router_split"], state["router_norms"],
                          cfg.k)
    pl = M.plan(ids, w, cfg.e)
    tiles = ((pl["counts"] + 511) // 512).to(torch.int32)
    mtile = torch.zeros(cfg.e + 1, dtype=torch.int32, device=x.device)
    mtile[1:] = torch.cumsum(tiles, 0)
    xp = M.gather_rows(x, pl["perm_slot"], div=cfg.k)
    for _ in range(3):
        M.expert_gate_up(xp, state["w_gate_up_packed"], pl["offsets"], mtile)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        M.expert_gate_up(xp, state["w_gate_up_packed"], pl["offsets"], mtile)
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return {"ms": statistics.mean(times), "flops": 4.0 * cfg.t * cfg.k * cfg.h * cfg.i}


def bench_moe(args, dist: Dist) -> dict | None:
    from kdb200 import moe as M
    from kdb200 import workloads as W

    cfg = W.MOE_CONFIGS[args.workload]
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    x = W.moe_input(cfg.t, cfg.h, seed=1 + dist.rank, device=dev)
    flush = _flusher(dev)
    holder = {}
    sampler = ClockSampler(_physical_index(dist.local)) if dist.rank == 0 else None
    ep = dist.world > 1
    state = None
    if ep:
        # Expert parallel: this rank's T tokens, its E/P experts; rows cross NVLink by NCCL all-to-all.
        from kdb200 import ep as EP
        er = cfg.e // dist.world
        wts = W.moe_weights(cfg, seed=1, device=dev, experts=range(dist.rank * er, (dist.rank + 1) * er))
        layer = EP.ExpertParallelMoE(wts, cfg.k, local_experts=True)
        del wts
        torch.cuda.empty_cache()

        def step():
            holder["out"] = layer(x)

        run_step = step
        forward = layer
    else:
        wts = W.moe_weights(cfg, seed=1, device=dev)
        state = M.prepare(wts, cfg.k)
        del wts
        torch.cuda.empty_cache()

        def step():
            holder["out"] = M.forward(x, state)

        run_step = _capture(step).replay
        sub = _load_submission("b200_moe_prefill")

        def forward(xx):
            return sub.kernel_fn({"x": xx, "config": cfg.as_case()}, state)
    per_step, region_ms = timed_steps(run_step, args.steps, args.warmup, flush, dist, sampler)
    ms = dist.max(statistics.mean(per_step))
    value = cfg.t * dist.world / (ms * 1e-3)
    ids = holder["out"][2]
    distinct = int(torch.unique(ids).numel())
    y_dev = holder["out"][0].clone()

    x_host = x.cpu().pin_memory()
    y_host = torch.empty((cfg.t, cfg.h), dtype=torch.bfloat16).pin_memory()
    w_host = torch.empty((cfg.t, cfg.k), dtype=torch.float32).pin_memory()
    i_host = torch.empty((cfg.t, cfg.k), dtype=torch.int32).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        y, w, i = forward(x_dev)
        y_host.copy_(y, non_blocking=True)
        w_host.copy_(w, non_blocking=True)
        i_host.copy_(i, non_blocking=True)

    e2e_steps, _ = timed_steps(e2e_step, max(3, args.steps // 4), 2, flush, dist, None)
    e2e_ms = dist.max(statistics.mean(e2e_steps))
    if not torch.equal(y_host.to(dev), y_dev):
        raise RuntimeError("e2e output differs from the device-resident run")
    dom = _time_dominant_gate_up(state, x, cfg, flush, max(3, args.steps // 2)) if state is not None else None
    if dist.rank != 0:
        return None
    peaks = _peaks()
    flops = W.moe_flops(cfg)                   # per rank: T tokens' routed work (weak scaling under EP)
    nbytes = W.moe_bytes(cfg, cfg.e // dist.world if ep else distinct)
    # each step is one flushed graph replay timed alone: the burst tensor peak applies
    t_c = flops / (peaks["bf16_tflops"] * 1e12)
    t_m = nbytes / (peaks["hbm_gbs"] * 1e9)
    layer_s = statistics.mean(per_step) * 1e-3
    bound = "tensor" if t_c >= t_m else "hbm"
    if bound == "tensor":
        ach = flops / layer_s / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4)}
    else:
        ach = nbytes / layer_s / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(ach / peaks["hbm_gbs"], 4)}
    traffic = _profile_traffic("moe_layer", args.workload)
    roof.update({"traffic": traffic, "peak_source": f"{peaks['source']} (burst: each step is timed alone)",
                 "kernel": "whole layer per graph replay (route, plan, gather, grouped gate_up, grouped down, "
                           "combine, shared expert)",
                 "algorithmic_flops": flops, "algorithmic_bytes": nbytes, "distinct_experts_hit": distinct,
                 "layer_roofline_ms": round(max(t_c, t_m) * 1e3, 4),
                 "frac_of_layer_roofline": round(max(t_c, t_m) / layer_s, 4)})
    if dom is not None:
        common = {"ms_per_launch": round(dom["ms"], 4), "traffic": _profile_traffic("moe_gate_up", args.workload),
                  "timing": "CUDA events around each launch after an untimed L2 flush"}
        if cfg.t > 64:
            dach = dom["flops"] / (dom["ms"] * 1e-3) / 1e12
            roof["dominant_kernel"] = {
                "kernel": "gemm_grouped_pair_kernel<GroupedPairSched, SwigluGpEpi> (routed gate_up + SwiGLU)",
                "bound": "tensor", "achieved": round(dach, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(dach / peaks["bf16_tflops"], 4), **common}
        else:
            gu_bytes = distinct * 2.0 * cfg.i * cfg.h * 2 + cfg.t * cfg.k * (cfg.h + cfg.i) * 2
            gbs = gu_bytes / (dom["ms"] * 1e-3) / 1e9
            roof["dominant_kernel"] = {
                "kernel": "gemm_swap_kernel<StreamSched, SwigluStreamEpi> (routed gate_up + SwiGLU, weight stream)",
                "bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(gbs / peaks["hbm_gbs"], 4), **common}
    launches = MOE_LAUNCHES_PER_CALL["base"] + (MOE_LAUNCHES_PER_CALL["ep"] if ep else 0) + \
        (MOE_LAUNCHES_PER_CALL["shared"] if cfg.shared else 0)
    if ep:
        path = "kdb200.ep.ExpertParallelMoE -> kdb_moe_* stage entry points + NCCL all_to_all_single"
    else:
        path = "submissions/b200_moe_prefill.py kernel_fn (kdev adapter API) -> kdb_moe_forward"
    line = {
        "metric": "MoE layer tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; x~N(0,1) bf16, router N(0,1/H) fp32, experts N(0,1/fan_in) bf16)",
        "config": _moe_config(cfg, dist.world, args.workload),
        "e2e": {"value": round(cfg.t * dist.world / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": cfg.t * cfg.h * 2,
                "d2h_bytes_per_step": cfg.t * cfg.h * 2 + cfg.t * cfg.k * 8,
                "path": path,
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": launches * args.steps,
        "roofline": roof,
        "clocks": sampler.summary() if sampler else None,
        "timed_region_ms": round(region_ms, 2),
    }
    if not args.no_cpu_baseline and dist.world == 1:
        line["cpu_baseline"] = cpu_baseline_moe(args.workload, seconds=args.cpu_seconds)
    return line


def _load_submission(name: str):
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        f"{name}_sub", ROOT / "kernel-development_b200" / "submissions" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# ------------------------------------------------------------------------------------------------ reference arm
def _proj_config(cfg, world: int, workload: str) -> dict:
    return {"workload": workload, "m": cfg.m, "k": cfg.k, "n_per_gpu": cfg.n, "n_total": cfg.n * world,
            "parallelism": f"column-parallel over N, {world} shard(s), no collective",
            "l2": "flushed before every timed step (512 MiB device write then read, untimed)",
            "graph": "CUDA graph replay per step"}


def _moe_config(cfg, world: int, workload: str) -> dict:
    if world > 1:
        par = (f"expert-parallel over {world} GPUs ({cfg.e // world} experts each, NCCL all-to-all "
               "dispatch and combine, weak scaling: T tokens per GPU)")
        graph = "eager (row split sizes read back to the host once per call)"
    else:
        par, graph = "1 GPU", "CUDA graph replay per step"
    return {"workload": workload, **cfg.as_case(), "parallelism": par,
            "l2": "flushed before every timed step (512 MiB device write then read, untimed)", "graph": graph}


def run_reference(args, dist) -> dict | None:
    """The reference arm: the path's PyTorch fp32 formulation (the oracle) on this host's cores, on the same
    workload, config, metric and unit as our arm; rank 0 only."""
    from kdb200 import workloads as W
    if dist.rank != 0:
        return None
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n = args.steps + args.warmup
    if args.workload.startswith("proj"):
        cfg = _proj_cfg(args.workload)
        b = cpu_baseline_proj(cfg, 0.0, steps=n)
        return {
            "impl": "reference", "metric": PROJ_METRIC, "value": b["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": _proj_config(cfg, world, args.workload),
            "cpu_baseline": b, "e2e": {"value": b["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                                       "d2h_bytes_per_step": 0}}
    if args.workload.startswith("attn"):
        b = cpu_baseline_attn(args.workload, steps=n)
        case, _ = W.ATTN_CONFIGS[args.workload]
        return {"impl": "reference", "metric": ATTN_METRIC, "value": b["value"], "unit": "keys/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.workload, **case}, "cpu_baseline": b,
                "e2e": {"value": b["value"], "unit": "keys/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload.startswith("w4a16"):
        b = cpu_baseline_w4a16(args.workload, steps=n)
        config = {"workload": args.workload}
    else:
        b = cpu_baseline_moe(args.workload, steps=n)
        config = _moe_config(W.MOE_CONFIGS[args.workload], world, args.workload)
    line = {"impl": "reference", "metric": "MoE layer tokens/s", "value": b["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
            "cpu_baseline": b, "e2e": {"value": b["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                       "d2h_bytes_per_step": 0}}
    if args.workload == DEFAULT_WORKLOAD and not args.no_projection:
        pcfg = _proj_cfg(NESTED_PROJ_WORKLOAD)
        pb = cpu_baseline_proj(pcfg, 0.0, steps=n)
        line["projection"] = {"metric": PROJ_METRIC, "value": pb["value"], "unit": "TFLOP/s",
                              "config": _proj_config(pcfg, world, NESTED_PROJ_WORKLOAD), "cpu_baseline": pb}
    return line


def cpu_baseline_moe(workload: str, seconds: float = 10.0, steps: int | None = None) -> dict:
    """The layer's PyTorch fp32 formulation on the host cores, costed per stage at the workload's real
    sizes and extrapolated to the whole batch:
      router  softmax(x.float() @ Wr.T (+ b)) -> top-k -> renormalised weights, on a token sample;
      routed  the oracle's SwiGLU expert (fp32 GEMMs from bf16 weights, bf16 intermediate) on sampled
              experts with all the tokens the full batch routes to them, plus the weighted index-add;
      shared  the shared expert on a token sample.
    tokens/s = 1 / (router s/token + k * routed s/route + shared s/token).  One evaluation runs each
    stage once; evaluations repeat until `seconds` (or `steps` evaluations) and the median is reported."""
    from kdb200 import workloads as W
    from oracle import moe as om

    cores = _cpu_threads()
    cfg = W.MOE_CONFIGS[workload]
    x = W.moe_input(cfg.t, cfg.h, seed=1)
    router = W._randn((cfg.e, cfg.h), 1 * 1000 + 3, "cpu", 1.0 / cfg.h ** 0.5, torch.float32)
    bias = W.zipf_router_bias(cfg.e, cfg.zipf_s, 1) if cfg.zipf_s > 0 else None
    # routing of the whole batch (untimed) gives each sampled expert its real token count
    lg = om.torch_fp32_logits(x, router, bias)
    ids_all = torch.topk(lg, cfg.k, dim=-1).indices
    counts = torch.bincount(ids_all.reshape(-1), minlength=cfg.e)
    order = torch.argsort(counts, descending=True)
    n_sample = 2 if cfg.e >= 2 else 1
    sample_experts = [int(order[len(order) // 2 + j]) for j in range(n_sample)]   # median-popularity experts
    sub_cfg = W.MoeConfig("cpu", cfg.t, cfg.h, cfg.e, cfg.i, cfg.k, cfg.shared, cfg.shared_i)
    wts = W.moe_weights(sub_cfg, seed=1, experts=sample_experts)
    rows_of = [(ids_all == e).any(dim=1).nonzero().flatten() for e in sample_experts]
    t_r = min(cfg.t, 256)
    xf = x.float()

    def evaluate() -> float:
        t0 = time.perf_counter()
        l = xf[:t_r] @ router.T
        if bias is not None:
            l = l + bias
        p = torch.softmax(l, dim=-1)
        v, _ = torch.topk(p, cfg.k, dim=-1)
        _ = v / v.sum(dim=-1, keepdim=True)
        s_router = (time.perf_counter() - t0) / t_r
        y = torch.zeros((cfg.t, cfg.h), dtype=torch.float32)
        t0 = time.perf_counter()
        routes = 0
        for j, rows in enumerate(rows_of):
            ye = om._expert(xf[rows], wts["w_gate_up"][j], wts["w_down"][j])
            y.index_add_(0, rows, ye * 0.125)
            routes += rows.numel()
        s_route = (time.perf_counter() - t0) / max(routes, 1)
        s_shared = 0.0
        if cfg.shared:
            t0 = time.perf_counter()
            om._expert(xf[:t_r], wts["shared_gate_up"][0], wts["shared_down"][0])
            s_shared = (time.perf_counter() - t0) / t_r
        return 1.0 / (s_router + cfg.k * s_route + s_shared)

    evaluate()   # warm-up
    rates, t_end = [], time.perf_counter() + seconds
    while (steps is None and (time.perf_counter() < t_end or len(rates) < 3)) or (steps is not None and len(rates) < steps):
        rates.append(evaluate())
    return {"value": round(statistics.median(rates), 2), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"PyTorch fp32 layer on the host: router on {t_r} of {cfg.t} tokens; experts "
                       f"{sample_experts} (median popularity) with all {sum(int(r.numel()) for r in rows_of)} "
                       f"routes the full batch sends them (oracle/moe.py _expert); shared expert on {t_r} tokens; "
                       f"extrapolated to {cfg.t} tokens x top-{cfg.k}; median of {len(rates)} evaluations")}


def cpu_baseline_w4a16(workload: str, steps: int = 3) -> dict:
    """Oracle NVFP4 w4a16 layer (oracle/moe_w4a16.py: dequantise, fp32 GEMMs, RMS norm) on the host cores
    over a bounded token sample, with the weights of the local experts that sample routes to."""
    from kdb200 import workloads as W
    from oracle import moe_w4a16 as ow

    cores = _cpu_threads()
    cfg = W.W4A16_CONFIGS[workload]
    ids, tw = W.w4a16_routing(cfg, 1)
    t_s = min(cfg.t, 16)
    ids, tw = ids[:t_s], tw[:t_s]
    hit = sorted({int(e) for e in ids.flatten().tolist() if int(e) < cfg.local})
    remap = {e: j for j, e in enumerate(hit)}
    sub = ids.clone().apply_(lambda e: remap.get(e, len(hit) + e))     # remote routes stay >= the local count
    wts = W.w4a16_weights(cfg, 1, experts=hit)
    x = W.moe_input(t_s, cfg.h, 1)
    rates = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        ow.w4a16_ref(x, sub, tw, wts, len(hit))
        rates.append(t_s / (time.perf_counter() - t0))
    return {"value": round(statistics.median(rates), 2), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{t_s} of {cfg.t} tokens through the layer ({len(hit)} local experts hit), "
                      f"oracle/moe_w4a16.py, median of {len(rates)}"}


# ------------------------------------------------------------------------------------------------ attention
ATTN_METRIC = "cached keys attended per second (keys x KV heads / s)"


def _attn_inputs(workload: str, device):
    from kdb200 import attention as A
    from kdb200 import workloads as W
    from oracle import attention as OA
    case, seed = W.ATTN_CONFIGS[workload]
    data = OA.generate_input(case, seed)
    window = A.window_of(case["layer"])
    return case, data, window, W.attn_keys(data, window)


def cpu_baseline_attn(workload: str, steps: int = 3) -> dict:
    """The oracle (oracle/attention.py: fp32 einsum over the appended cache) on the host cores, on the first
    sequence of the workload's batch (a bounded sample), in the same unit."""
    from kdb200 import workloads as W
    from oracle import attention as OA
    cores = _cpu_threads()
    case, data, window, _ = _attn_inputs(workload, "cpu")
    one = {k: (v[:1] if isinstance(v, torch.Tensor) and k not in ("k_cache", "v_cache") else v)
           for k, v in data.items()}
    one["k_cache"], one["v_cache"] = data["k_cache"], data["v_cache"]
    keys = W.attn_keys(one, window)
    rates = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        OA.attention_ref(one)
        rates.append(keys / (time.perf_counter() - t0))
    return {"value": round(statistics.median(rates), 1), "unit": "keys/s", "cores": cores, "kind": "port",
            "sample": f"sequence 0 of {case['batch']} ({keys} keys x KV heads), oracle/attention.py attention_ref "
                      f"(append + fp32 einsum softmax), median of {len(rates)}"}


def bench_attn(args, dist: Dist) -> dict | None:
    """FP8-KV paged decode / verify attention, one call per step (append + attention + merge), one GPU."""
    from kdb200 import attention as A
    if dist.world > 1:
        raise SystemExit("attention workloads run on one GPU (replicas only): use --gpus 1")
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    case, data, window, keys = _attn_inputs(args.workload, dev)
    g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in data.items()}
    flush = _flusher(dev)
    holder = {}
    sampler = ClockSampler(_physical_index(dist.local))

    def call(q, kn, vn, bt, sl):
        return A.decode(q, kn, vn, g["k_cache"], g["v_cache"], bt, sl, data["kv_scale"], window)

    def step():
        holder["out"] = call(g["q"], g["k_new"], g["v_new"], g["block_table"], g["seq_lens"])

    run_step = _capture(step).replay
    per_step, region_ms = timed_steps(run_step, args.steps, args.warmup, flush, dist, sampler)
    ms = statistics.mean(per_step)
    # the attention kernel alone, on the same stream (events around it inside an eager call are not possible
    # without splitting the op, so time the whole call and report the kernel share from the ncu launch list)
    T = data["q"].shape[1]
    small = data["q"].numel() * 2 * 2 + data["k_new"].numel() * 2 * 2 + data["k_new"].numel() * 2
    nbytes = keys * 256 + small + data["block_table"].numel() * 4
    host = {k: g[k].cpu().pin_memory() for k in ("q", "k_new", "v_new", "block_table", "seq_lens")}
    devbuf = {k: torch.empty_like(g[k]) for k in host}
    out_host = torch.empty(tuple(data["q"].shape), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        for k in host:
            devbuf[k].copy_(host[k], non_blocking=True)
        out_host.copy_(call(devbuf["q"], devbuf["k_new"], devbuf["v_new"], devbuf["block_table"],
                            devbuf["seq_lens"]), non_blocking=True)

    e2e_steps, _ = timed_steps(e2e_step, max(3, args.steps // 4), 3, flush, dist, None)
    e2e_ms = statistics.mean(e2e_steps)
    h2d = sum(int(v.numel() * v.element_size()) for v in host.values())
    peaks = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": ATTN_METRIC, "value": round(keys / (ms * 1e-3), 1), "unit": "keys/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 cache x (q, p as two e4m3 terms), fp32 acc",
        "data": "synthetic (seeded oracle/attention.py generator; the reference problem's case and seed)",
        "config": {"workload": args.workload, **case, "window": window, "keys_x_kv_heads": keys,
                   "parallelism": "1 GPU (replicas only)",
                   "l2": "flushed before every timed step (512 MiB device write then read, untimed)",
                   "graph": "CUDA graph replay per step"},
        "e2e": {"value": round(keys / (e2e_ms * 1e-3), 1), "unit": "keys/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": int(out_host.numel() * 2), "ms_per_step": round(e2e_ms, 5),
                "path": "kdb200.attention.decode -> kdb_attn_decode_fp8 (q, k_new, v_new, block_table, seq_lens "
                        "copied in; the cache stays resident)"},
        "gpu_launches": 3 * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": f"{peaks['source']} (burst)",
                     "kernel": "whole call (append, attention, merge); bytes = 256 B per cached key and KV head "
                               "+ q, k_new, v_new, out, block table"},
        "clocks": sampler.summary(),
        "timed_region_ms": round(region_ms, 3),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_attn(args.workload)
    return line


# ------------------------------------------------------------------------------------------------ main
def bench_w4a16(args, dist: Dist) -> dict | None:
    """NVFP4 w4a16 MoE layer of one ep8 rank (1 GPU; the layer is one rank's slice by definition)."""
    from kdb200 import moe_w4a16 as W4
    from kdb200 import workloads as W
    if dist.world > 1:
        raise SystemExit("w4a16 workloads are one expert-parallel rank's layer: run them with --gpus 1")
    cfg = W.W4A16_CONFIGS[args.workload]
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    state = W4.prepare(W.w4a16_weights(cfg, 1), dev)
    ids, tw = W.w4a16_routing(cfg, 1)
    x = W.moe_input(cfg.t, cfg.h, 1, device=dev)
    gi, gw = ids.to(dev), tw.to(dev)
    flush = _flusher(dev)
    holder = {}
    sampler = ClockSampler(_physical_index(dist.local))

    def step():
        holder["y"] = W4.forward(x, gi, gw, state, cfg.e_total)

    run_step = _capture(step).replay
    per_step, region_ms = timed_steps(run_step, args.steps, args.warmup, flush, dist, sampler)
    ms = statistics.mean(per_step)
    hit = sorted({int(e) for e in ids.flatten().tolist() if int(e) < cfg.local})
    per_expert = 3 * cfg.h * cfg.i * (0.5 + 1.0 / 16)        # E2M1 codes + E4M3 scales
    nbytes = len(hit) * per_expert + cfg.t * cfg.h * 4 + cfg.t * cfg.k * 8
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((cfg.t, cfg.h), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        y_host.copy_(W4.forward(x_dev, gi, gw, state, cfg.e_total), non_blocking=True)

    e2e_steps, _ = timed_steps(e2e_step, max(3, args.steps // 4), 2, flush, dist, None)
    e2e_ms = statistics.mean(e2e_steps)
    peaks = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {
        "metric": "MoE layer tokens/s", "value": round(cfg.t / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 weights x bf16 activations (f16 operands), fp32 acc",
        "data": "synthetic (seeded; x~N(0,1) bf16, experts N(0,1/fan_in) quantised to NVFP4, routing with this "
                "rank the busiest)",
        "config": {"workload": args.workload, "t": cfg.t, "h": cfg.h, "i": cfg.i, "local_experts": cfg.local,
                   "e_total": cfg.e_total, "k": cfg.k, "local_experts_hit": len(hit),
                   "parallelism": "one ep8 rank's slice on 1 GPU",
                   "l2": "flushed before every timed step (512 MiB device write then read, untimed)",
                   "graph": "CUDA graph replay per step"},
        "e2e": {"value": round(cfg.t / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "h2d_bytes_per_step": cfg.t * cfg.h * 2,
                "d2h_bytes_per_step": cfg.t * cfg.h * 2, "path": "kdb200.moe_w4a16.forward -> kdb_moe_w4a16_forward",
                "ms_per_step": round(e2e_ms, 4)},
        # plan (3), tile prefix, gather, gate_up, down, combine
        "gpu_launches": 8 * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": f"{peaks['source']} (burst)",
                     "kernel": "whole layer (plan, gather, NVFP4 gate_up, NVFP4 down, RMS-norm combine); "
                               "bytes = NVFP4 weights of the local experts hit + activations"},
        "clocks": sampler.summary(),
        "timed_region_ms": round(region_ms, 3),
    }


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-projection", action="store_true",
                    help=f"default workload only: skip the nested {NESTED_PROJ_WORKLOAD} projection record")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        line = run_reference(args, _RefDist())
        print(json.dumps(line), flush=True)
        return 0
    dist = Dist()
    try:
        if args.workload.startswith("proj"):
            line = bench_proj(args, dist)
        elif args.workload.startswith("moe"):
            line = bench_moe(args, dist)
            if args.workload == DEFAULT_WORKLOAD and not args.no_projection:
                # the projection headline of the same run, nested so one line carries both paths
                torch.cuda.empty_cache()
                pargs = argparse.Namespace(**{**vars(args), "workload": NESTED_PROJ_WORKLOAD})
                pline = bench_proj(pargs, dist)
                if line is not None and pline is not None:
                    for key in ("n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline"):
                        pline.pop(key, None)
                    line["projection"] = pline
        elif args.workload.startswith("w4a16"):
            line = bench_w4a16(args, dist)
        elif args.workload.startswith("attn"):
            line = bench_attn(args, dist)
        else:
            raise SystemExit(f"unknown workload {args.workload}")
        if line is not None and dist.rank == 0:
            if dist.world > 1:
                line.pop("cpu_baseline", None)
                if "projection" in line:
                    line["projection"].pop("cpu_baseline", None)
            print(json.dumps(line), flush=True)
    finally:
        dist.close()
    return 0


class _RefDist:
    rank = 0
    world = 1
    local = 0


if __name__ == "__main__":
    sys.exit(main())
