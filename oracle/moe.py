"""The MoE layer restated in numpy (oracle; test infrastructure only).

Router: dsv41/tt/moe.py:108-125 (fp32 logits, score function, bias used only for selection,
unbiased weights gathered at the chosen indices, ``/ (sum + 1e-20) * route_scale``).
Expert FFN: dsv41/tt/moe.py:133-139 (gate clamped <= 10, up clamped to [-10, 10], SiLU(gate)*up,
routing weight applied BEFORE w2). Routed + shared summed before the all-reduce:
dsv41/tt/moe.py:162, 180. Per-linear arithmetic: dsv41/ref/kernel.py:101-112 (fp32 dequantized
weights, activations promoted to fp32).

Reduction order is not part of the reference's algorithm, so the oracle pins it away: every dot
product is accumulated in float64 (each fp32 x bf16 product is exact there) and rounded once.
The CUDA router does the same, so router logits agree to the last bit and the top-k indices are
bit-exact except on exact ties, which both sides break toward the lower expert index.
"""
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from .formats import bf16_round, dequant_fp4, dequant_fp8_block

LIMIT = 10.0        # SwiGLU clamp (dsv41/tt/moe.py:15)
SCORE_FUNCS = ("sigmoid", "sqrtsoftplus")


# ---------------------------------------------------------------- router

def router_logits(x: np.ndarray, wg: np.ndarray) -> np.ndarray:
    """x [B, H] (bf16 values as float32) @ wg[E, H]^T -> fp32 [B, E], float64 accumulation."""
    return (np.asarray(x, np.float64) @ np.asarray(wg, np.float64).T).astype(np.float32)


def score(logits: np.ndarray, func: str) -> np.ndarray:
    """score function in float64, rounded once to fp32.

    sqrtsoftplus = sqrt(softplus(l)) as in dsv41/tt/moe.py:121 (torch softplus returns l itself
    above the threshold 20); sigmoid is the benchmark configuration's score function.
    """
    l = np.asarray(logits, np.float64)
    if func == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-l))
    elif func == "sqrtsoftplus":
        sp = np.where(l > 20.0, l, np.log1p(np.exp(np.minimum(l, 20.0))))
        s = np.sqrt(sp)
    else:
        raise ValueError(func)
    return s.astype(np.float32)


def topk_lower_index(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values per row, descending; ties go to the lower index."""
    v = np.asarray(v, np.float32)
    b, e = v.shape
    order = np.lexsort((np.broadcast_to(np.arange(e), v.shape), -v.astype(np.float64)), axis=-1)
    return order[:, :k].astype(np.int64)


def route(x, wg, bias, topk=6, score_func="sigmoid", route_scale=2.5,
          bias_vl=None, image_mask=None):
    """(idx [B,k] int64, wt [B,k] fp32, sc [B,E] fp32) -- dsv41/tt/moe.py:120-125."""
    logits = router_logits(x, wg)
    sc = score(logits, score_func)
    b = np.broadcast_to(np.asarray(bias, np.float32), sc.shape)
    if bias_vl is not None and image_mask is not None:
        b = np.where(np.asarray(image_mask, bool)[:, None], np.asarray(bias_vl, np.float32), b)
    biased = (sc + b).astype(np.float32)
    idx = topk_lower_index(biased, topk)
    wt = np.take_along_axis(sc, idx, axis=1).astype(np.float32)
    tot = np.zeros(wt.shape[0], np.float32)
    for j in range(topk):                       # sequential fp32 sum in top-k order
        tot = (tot + wt[:, j]).astype(np.float32)
    wt = (wt / (tot[:, None] + np.float32(1e-20)) * np.float32(route_scale)).astype(np.float32)
    return idx, wt, sc


def near_tie(x, wg, bias, topk=6, score_func="sigmoid", eps=1e-6) -> np.ndarray:
    """Per token: True when the k-th and (k+1)-th biased scores are within eps (index may flip)."""
    sc = score(router_logits(x, wg), score_func)
    biased = np.sort((sc + np.asarray(bias, np.float32)).astype(np.float64), axis=1)[:, ::-1]
    return (biased[:, topk - 1] - biased[:, topk]) < eps


# ---------------------------------------------------------------- experts

@dataclass
class QuantExpert:
    """One expert in the reference's checkpoint layout ([out, in] row-major).

    fmt "fp8": w* uint8 e4m3 codes, s* fp32 128x128-block scales.
    fmt "fp4": w* uint8 packed e2m1 [out, in/2], s* uint8 e8m0 [out, in/32].
    """
    fmt: str
    w1: np.ndarray
    s1: np.ndarray
    w3: np.ndarray
    s3: np.ndarray
    w2: np.ndarray
    s2: np.ndarray
    _cache: dict = field(default_factory=dict, repr=False)

    def dense(self, name: str) -> np.ndarray:
        """fp32 dequantized [out, in] (dsv41/ref/kernel.py:75-78 or 91-98)."""
        if name not in self._cache:
            w, s = getattr(self, name), getattr(self, "s" + name[1:])
            self._cache[name] = dequant_fp8_block(w, s) if self.fmt == "fp8" else dequant_fp4(w, s)
        return self._cache[name]


def silu(v):
    return v / (1.0 + np.exp(-v))


def expert_ffn(x: np.ndarray, e: QuantExpert, wt: Optional[np.ndarray] = None,
               rows: Optional[slice] = None, mimic_bf16: bool = False) -> np.ndarray:
    """dsv41/tt/moe.py:133-139 for tokens x [T, H]; returns the (partial) output [T, H] in float64.

    ``rows`` restricts the intermediate dimension to one tensor-parallel slice (w1/w3 rows and the
    matching w2 columns, dsv41/tt/moe.py:2-3), giving that rank's partial sum.
    ``mimic_bf16`` rounds each linear output and the SwiGLU result to bf16, as the reference's
    ``fp8_gemm``/``fp4_gemm`` return the default dtype (bf16) (dsv41/ref/kernel.py:105-112).
    """
    rows = rows or slice(None)
    x64 = np.asarray(x, np.float64)
    w1 = e.dense("w1")[rows].astype(np.float64)
    w3 = e.dense("w3")[rows].astype(np.float64)
    w2 = e.dense("w2")[:, rows].astype(np.float64)
    g = x64 @ w1.T
    u = x64 @ w3.T
    if mimic_bf16:
        g = bf16_round(g.astype(np.float32)).astype(np.float64)
        u = bf16_round(u.astype(np.float32)).astype(np.float64)
    g = np.minimum(g, LIMIT)
    u = np.clip(u, -LIMIT, LIMIT)
    h = silu(g) * u
    if wt is not None:
        h = h * np.asarray(wt, np.float64)[:, None]
    if mimic_bf16:
        h = bf16_round(h.astype(np.float32)).astype(np.float64)
    y = h @ w2.T
    if mimic_bf16:
        y = bf16_round(y.astype(np.float32)).astype(np.float64)
    return y


@dataclass
class MoELayer:
    """One MoE layer's weights in the reference layout (oracle side)."""
    wg: np.ndarray                  # [E, H] fp32 router weight
    bias: np.ndarray                # [E] fp32
    experts: list                   # E QuantExpert (routed)
    shared: QuantExpert             # the shared expert
    topk: int = 6
    score_func: str = "sigmoid"
    route_scale: float = 2.5
    bias_vl: Optional[np.ndarray] = None


def moe_forward(layer: MoELayer, x: np.ndarray, rank: int = 0, world: int = 1,
                mimic_bf16: bool = False, image_mask=None, return_partial: bool = False):
    """Routed + shared experts for tokens x [B, H] (bf16 values in float32).

    With world > 1 this is rank ``rank``'s partial (its 1/world slice of every expert's
    intermediate dimension); summing the partials over ranks is the all-reduce
    (dsv41/tt/attn.py:19-21). Returns (y [B, H] float64 -- rounded to bf16 unless
    ``return_partial`` --, idx, wt).
    """
    idx, wt, _ = route(x, layer.wg, layer.bias, layer.topk, layer.score_func, layer.route_scale,
                       layer.bias_vl, image_mask)
    inter = layer.shared.dense("w1").shape[0]
    assert inter % world == 0
    sl = slice(rank * inter // world, (rank + 1) * inter // world)
    y = expert_ffn(x, layer.shared, None, sl, mimic_bf16)
    for e in np.unique(idx):
        tok, kk = np.nonzero(idx == e)
        y[tok] += expert_ffn(x[tok], layer.experts[int(e)], wt[tok, kk], sl, mimic_bf16)
    if return_partial:
        return y, idx, wt
    return bf16_round(y.astype(np.float32)).astype(np.float64), idx, wt


def moe_forward_routed(layer: MoELayer, x: np.ndarray, idx: np.ndarray, wt: np.ndarray, rank: int = 0,
                       world: int = 1, return_partial: bool = False) -> np.ndarray:
    """The layer for tokens x [P, H] with routing given (idx [P, k], wt [P, k]): the batched prefill
    of dsv41/tt/moe.py:182-200, 263-288 (bincount, per-expert buckets, gather, FFN, weighted
    scatter-add) computes exactly this sum; the shared expert takes every token."""
    inter = layer.shared.dense("w1").shape[0]
    sl = slice(rank * inter // world, (rank + 1) * inter // world)
    y = expert_ffn(x, layer.shared, None, sl)
    for e in np.unique(idx):
        tok, kk = np.nonzero(idx == e)
        y[tok] += expert_ffn(x[tok], layer.experts[int(e)], wt[tok, kk], sl)
    if return_partial:
        return y
    return bf16_round(y.astype(np.float32)).astype(np.float64)


def compare(y: np.ndarray, y_ref: np.ndarray):
    """(max-abs-rel, cosine): max|y - ref| / max|ref| and the cosine similarity of the flattened rows."""
    y = np.asarray(y, np.float64).ravel()
    r = np.asarray(y_ref, np.float64).ravel()
    mar = float(np.max(np.abs(y - r)) / max(np.max(np.abs(r)), 1e-30))
    cos = float(np.dot(y, r) / max(np.linalg.norm(y) * np.linalg.norm(r), 1e-300))
    return mar, cos
