"""Comparison side for kdev's judge-mode timing of this problem (`kdev time --judge-mode` loads baseline.py from
the problem dir as the in-process baseline, src/kdev/timing/engine.py:960-984): the projection through
torch.matmul (cuBLAS) in bf16, the fp32 router layer through an fp32 matmul.  TEST INFRASTRUCTURE, never the
product."""
import torch


def prepare(weights):
    return {k: w.contiguous() for k, w in weights.items()}


def kernel_fn(data, state):
    w = state[data["config"]["layer"]]
    if w.dtype == torch.float32:
        return data["x"].float() @ w.t()
    return data["x"] @ w.t()
