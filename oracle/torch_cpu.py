"""The torch-CPU evaluation of BASELINE.json's configurations (the reported CPU baseline).

TEST / BASELINE INFRASTRUCTURE ONLY: ``bench.py`` times these on the host cores (its
``cpu_baseline`` leg and its ``--impl reference`` arm); nothing in the product imports it.

The reference defines every problem as a torch expression evaluated on the CPU by its
harness (``tools/generate.py:2``, the ``code=`` field of each problem, e.g.
``tests/expressions_quant.py:39-40`` for the bf16 matmul, ``tests/expressions_extra.py:412``
for ``scaled_dot_product_attention``, ``tests/expressions_llm.py:76-77`` for the weighted
RMSNorm with eps 1e-6, ``tools/expressions_open.py`` for softmax and sums).  These are
those expressions at the BASELINE configurations, computed as torch computes them on
the CPU: bf16 operands for the bf16 matmul and attention, f32 elsewhere, the FP8 GEMM as
e4m3-valued operands multiplied in f32 and scaled into bf16.  torch runs with every
host thread (``torch.set_num_threads(os.cpu_count())``).
"""

from __future__ import annotations

import os

import numpy as np


def threads() -> int:
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def sample_fn(name: str, inputs: dict):
    """A callable that evaluates the configuration's torch expression on the sample
    ``inputs`` (``baseline_configs.cpu_sample_inputs``)."""
    import torch
    import torch.nn.functional as F
    t = torch.from_numpy
    if name.startswith("gemm"):
        a = t(inputs["A"]).to(torch.bfloat16)
        b = t(inputs["B"]).to(torch.bfloat16)
        return lambda: a @ b
    if name == "fp8_8192":
        A, B = t(inputs["A"]), t(inputs["B"])
        # per-tensor scales amax / 448 over the whole operands (the sample holds all of B;
        # A's scale comes from its sampled rows, which only sets the sample's values)
        sa, sb = A.abs().max() / 448.0, B.abs().max() / 448.0
        aq = (A / sa).to(torch.float8_e4m3fn).float()
        bq = (B / sb).to(torch.float8_e4m3fn).float()
        scale = sa * sb
        return lambda: ((aq @ bq) * scale).to(torch.bfloat16)
    if name == "attention":
        q, k, v = (t(inputs[r]).to(torch.bfloat16) for r in ("Q", "K", "V"))
        return lambda: F.scaled_dot_product_attention(q, k, v)
    if name == "rmsnorm":
        x, w = t(inputs["X"]), t(inputs["W"])
        return lambda: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    if name == "softmax":
        x = t(inputs["X"])
        return lambda: torch.softmax(x, -1)
    if name == "sum":
        x = t(inputs["X"])
        return lambda: x.sum()
    raise KeyError(name)


def result_as_numpy(r) -> np.ndarray:
    import torch
    return r.float().numpy() if r.dtype != torch.float32 else r.numpy()
