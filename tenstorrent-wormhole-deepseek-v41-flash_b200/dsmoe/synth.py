"""Seeded synthetic weights and inputs in the benchmark configurations' formats.

Weights are drawn N(0, 0.02) in fp32 and quantized either to FP8 e4m3 with one fp32 scale per
128x128 block (scale = blockmax / 448) or to FP4 e2m1 (two per byte, low nibble first) with one
e8m0 scale per 32 K values (scale = pow2ceil(max(amax, 6 * 2^-126) / 6), values rounded to the e2m1
grid with ties to the even code) -- the quantizer rules of dsv41/ref/kernel.py:15-29, 69-70.
The same torch code runs on CPU (tests, bit-identical to the numpy oracle's quantizers) or on the
GPU (full-size benchmark layers, generated in HBM).
"""
from dataclasses import dataclass
from typing import Optional

import torch

FP4_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def quant_fp8_block(w: torch.Tensor, block: int = 128):
    """fp32 [N, K] -> (uint8 e4m3 codes [N, K], fp32 scales [ceil(N/b), ceil(K/b)])."""
    n, k = w.shape
    nb, kb = -(-n // block), -(-k // block)
    if n % block or k % block:
        pad = torch.zeros(nb * block, kb * block, device=w.device, dtype=torch.float32)
        pad[:n, :k] = w
    else:
        pad = w.float()
    s = pad.abs().view(nb, block, kb, block).amax(dim=(1, 3)).clamp(min=1e-30) / 448.0
    srep = s.repeat_interleave(block, 0)[:n].repeat_interleave(block, 1)[:, :k]
    q = (w / srep).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), s.float().contiguous()


def _pow2_ceil(x: torch.Tensor) -> torch.Tensor:
    m, e = torch.frexp(x.float())
    return torch.ldexp(torch.ones_like(m), torch.where(m == 0.5, e - 1, e))


def quant_fp4_e8m0(w: torch.Tensor, group: int = 32):
    """fp32 [N, K] -> (uint8 packed e2m1 [N, K/2], uint8 e8m0 [N, K/32])."""
    n, k = w.shape
    wb = w.float().view(n, k // group, group)
    amax = wb.abs().amax(-1, keepdim=True)
    s = _pow2_ceil(amax.clamp(min=6 * 2.0 ** -126) / 6.0)
    v = wb / s
    grid = torch.tensor(FP4_GRID, device=w.device)
    a = v.abs().clamp(max=6.0)
    hi = torch.searchsorted(grid, a.contiguous()).clamp(max=7)
    lo = (hi - 1).clamp(min=0)
    dlo, dhi = a - grid[lo], grid[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    mag = torch.where(pick_hi, hi, lo).to(torch.uint8)
    code = (mag | (((v < 0) & (mag > 0)).to(torch.uint8) << 3)).view(n, k)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
    e8 = (torch.frexp(s)[1] - 1 + 127).to(torch.uint8).view(n, k // group).contiguous()
    return packed, e8


@dataclass
class ExpertWeights:
    """One expert in the checkpoint layout: w1/w3 [I, H], w2 [H, I] (quantized), and their scales."""
    fmt: str
    w1: torch.Tensor
    s1: torch.Tensor
    w3: torch.Tensor
    s3: torch.Tensor
    w2: torch.Tensor
    s2: torch.Tensor

    def to(self, device):
        return ExpertWeights(self.fmt, *(getattr(self, n).to(device) for n in ("w1", "s1", "w3", "s3", "w2", "s2")))


def make_expert(fmt: str, hidden: int, inter: int, gen: torch.Generator, device="cpu", std=0.02) -> ExpertWeights:
    out = []
    for shape in ((inter, hidden), (inter, hidden), (hidden, inter)):
        w = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std
        out.extend(quant_fp8_block(w) if fmt == "fp8" else quant_fp4_e8m0(w))
        del w
    return ExpertWeights(fmt, *out)


@dataclass
class RouterWeights:
    wg: torch.Tensor          # [E, H] fp32
    bias: torch.Tensor        # [E] fp32
    bias_vl: Optional[torch.Tensor] = None


def make_router(n_experts: int, hidden: int, gen: torch.Generator, device="cpu", std=0.02, bias_std=0.01):
    wg = torch.randn((n_experts, hidden), generator=gen, device=device, dtype=torch.float32) * std
    bias = torch.randn((n_experts,), generator=gen, device=device, dtype=torch.float32) * bias_std
    return RouterWeights(wg, bias)


def make_tokens(n: int, hidden: int, gen: torch.Generator, device="cpu") -> torch.Tensor:
    return torch.randn((n, hidden), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def zipf_routing(n_tokens: int, n_experts: int, topk: int, gen: torch.Generator, s: float = 1.1,
                 route_scale: float = 2.5):
    """Skewed routing for the prefill benchmark: expert popularity ~ Zipf(s) over a seeded random
    permutation of the experts, each token drawing ``topk`` distinct experts without replacement;
    weights uniform in [0.5, 1.5), normalised to sum to ``route_scale`` per token.
    Returns (idx [n, k] int64, wt [n, k] float32) on the CPU."""
    ranks = torch.arange(1, n_experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    perm = torch.randperm(n_experts, generator=gen)
    probs = torch.empty(n_experts, dtype=torch.float64)
    probs[perm] = p
    idx = torch.multinomial(probs.expand(n_tokens, -1).contiguous(), topk, replacement=False, generator=gen)
    w = torch.rand((n_tokens, topk), generator=gen, dtype=torch.float32) + 0.5
    wt = w / w.sum(dim=1, keepdim=True) * route_scale
    return idx.to(torch.int64), wt.to(torch.float32)
