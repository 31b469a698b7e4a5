"""The reference's CPU path for one MoE layer, timed as the benchmark's CPU baseline
(test infrastructure: only bench.py's CPU-baseline leg and ``--impl reference`` use it).

What runs per layer and step, following the reference line by line on torch CPU tensors:
* router: fp32 ``x.float() @ Wg^T`` (the Gate's linear), score function, bias for selection only,
  top-k, gathered weights ``/ (sum + 1e-20) * route_scale`` (dsv41/tt/moe.py:108-125);
* each of the k routed experts and the shared expert through the shim's linears with
  ``DSV41_FAKEQUANT=0``: ``act_quant`` passes activations through as fp32, the weight is
  dequantized to fp32 on every call (``_deq_fp8_weight``, dsv41/ref/kernel.py:75-78, or
  ``dequant_fp4_weight``, :91-98 -- through the reference's own fp4lib.c when it is built, as the
  shim does), ``a @ w.T`` in fp32, output rounded to bf16 (dsv41/ref/kernel.py:101-112);
* the FFN: gate clamped <= 10, up clamped to +-10, SiLU(gate) * up, routing weight before w2
  (dsv41/tt/moe.py:133-139), routed + shared summed (dsv41/tt/moe.py:162, 180).

Threads: all the cores torch may use (``torch.set_num_threads`` = the affinity mask size).
"""
import os
import platform
import time

import torch

from . import ref_fp4lib


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def use_all_cores() -> int:
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


_FP4_TABLE = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _deq_fp8(q_u8: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    n, k = q_u8.shape
    sr = s.float().repeat_interleave(128, 0)[:n].repeat_interleave(128, 1)[:, :k]
    return q_u8.view(torch.float8_e4m3fn).float() * sr


def _deq_fp4(q_u8: torch.Tensor, s_u8: torch.Tensor) -> torch.Tensor:
    if ref_fp4lib.available():
        return torch.from_numpy(ref_fp4lib.dequant_fp4(q_u8.numpy(), s_u8.numpy()))
    idx = torch.stack([q_u8 & 0x0F, q_u8 >> 4], dim=-1).flatten(-2).long()
    return _FP4_TABLE[idx] * s_u8.view(torch.float8_e8m0fnu).float().repeat_interleave(32, dim=-1)


def linear(x_bf16: torch.Tensor, fmt: str, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    w = _deq_fp8(q, s) if fmt == "fp8" else _deq_fp4(q, s)
    return (x_bf16.float() @ w.T).to(torch.bfloat16)


def ffn(x, ew, wt=None):
    g = linear(x, ew.fmt, ew.w1, ew.s1).clamp(max=10.0)
    u = linear(x, ew.fmt, ew.w3, ew.s3).clamp(min=-10.0, max=10.0)
    h = torch.nn.functional.silu(g) * u
    if wt is not None:
        h = h * wt.to(h.dtype).unsqueeze(-1)
    return linear(h, ew.fmt, ew.w2, ew.s2)


def layer(x, wg, bias, experts_of, shared, topk=6, route_scale=2.5):
    """One MoE layer; ``experts_of(e)`` returns routed expert e's checkpoint-layout weights."""
    logits = x.float() @ wg.T
    sc = torch.sigmoid(logits)
    idx = (sc + bias).topk(topk, dim=-1).indices
    wt = sc.gather(1, idx)
    wt = wt / (wt.sum(-1, keepdim=True) + 1e-20) * route_scale
    y = ffn(x, shared).float()
    for e in idx.unique().tolist():
        tok, kk = torch.where(idx == e)
        y[tok] += ffn(x[tok], experts_of(e), wt[tok, kk]).float()
    return y.to(torch.bfloat16)


def time_steps(step_fn, steps: int, warmup: int, min_steps: int = 1, budget_s: float = None):
    """Run ``warmup`` untimed steps, then ``steps`` timed (or fewer if ``budget_s`` runs out,
    never below ``min_steps``). Returns (seconds per step, steps timed)."""
    for i in range(warmup):
        step_fn(i)
    t0 = time.perf_counter()
    n = 0
    while n < steps:
        step_fn(warmup + n)
        n += 1
        if budget_s is not None and n >= min_steps and time.perf_counter() - t0 > budget_s:
            break
    return (time.perf_counter() - t0) / n, n
