"""CUDA drop-in for the operator module DeepSeek-V4.1-Flash's ``inference/model.py`` imports as
``kernel`` -- the surface the reference shims on the CPU in dsv41/ref/kernel.py and puts on
``sys.path`` ahead of the model (dsv41/ref/load.py:12-14). Put this directory first on ``sys.path``
the same way and the model's ``import kernel`` gets B200 kernels.

Same names, signatures and return dtypes as the shim (dsv41/ref/kernel.py:44, 58, 91, 105, 110),
plus ``weight_dequant`` (the FP8 block dequant entry point of DeepSeek's kernel module).
``DSV41_FAKEQUANT`` has the shim's meaning and default (dsv41/ref/kernel.py:36-41): "0" keeps
activations exact, anything else fake-quantizes linear inputs to e4m3 per 128.

Inputs must be CUDA tensors: there is no CPU path. ``sparse_attn`` and ``hc_split_sinkhorn``
belong to attention and hyper-connections, which this package does not implement.
"""
import os as _os

import torch

from dsmoe import _lib as _L

FAKEQUANT = _os.environ.get("DSV41_FAKEQUANT", "1") != "0"


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("dsmoe kernels take CUDA tensors only")


def _u8(t):
    return t.contiguous().view(torch.uint8)


def act_quant(x, block_size=128, scale_fmt=None, scale_dtype=torch.float32, inplace=False):
    """dsv41/ref/kernel.py:44-55."""
    assert x.size(-1) % block_size == 0
    if not FAKEQUANT:
        return x if inplace else (x.float(), torch.ones(*x.shape[:-1], x.size(-1) // block_size, device=x.device))
    _cuda(x)
    x2 = x.reshape(-1, x.size(-1)).contiguous()
    if x2.dtype not in (torch.float32, torch.bfloat16):
        x2 = x2.float()
    M, K = x2.shape
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((M, K // block_size), dtype=torch.float32, device=x.device)
    _L.call("dsmoe_act_quant", _L.ptr(x2), _L.DTYPE_F32 if x2.dtype == torch.float32 else _L.DTYPE_BF16, M, K,
            block_size, 1 if scale_fmt is not None else 0, _L.ptr(q), _L.ptr(s), _L.stream_of(x2))
    q8 = q.view(torch.float8_e4m3fn)
    if inplace:
        deq = (q8.float().view(M, K // block_size, block_size) * s.unsqueeze(-1)).view(M, K)
        x.copy_(deq.view(x.shape).to(x.dtype))
        return x
    return q8.view(*x.shape), s.view(*x.shape[:-1], K // block_size).to(scale_dtype)


def fp4_act_quant(x, block_size=32, inplace=False, scale_dtype=torch.float8_e8m0fnu):
    """dsv41/ref/kernel.py:58-72; only the exact-activation mode is on the MoE path."""
    assert scale_dtype in (torch.float8_e8m0fnu, torch.float8_e4m3fn)
    assert x.size(-1) % block_size == 0
    if not inplace:
        raise NotImplementedError("packed FP4 output is unused by model.py; only inplace is provided")
    if not FAKEQUANT:
        return x
    raise NotImplementedError("FP4 activation fake-quant serves attention (indexer / compressed KV), "
                              "which this package does not implement")


def _gemm(fn, a, a_s, b, b_s, block):
    _cuda(a, a_s, b, b_s)
    K = a.size(-1)
    a2 = a.reshape(-1, K)
    if a2.dtype == torch.float8_e4m3fn:
        adt, a2 = _L.DTYPE_E4M3, a2.contiguous().view(torch.uint8)
    elif a2.dtype == torch.bfloat16:
        adt, a2 = _L.DTYPE_BF16, a2.contiguous()
    else:
        adt, a2 = _L.DTYPE_F32, a2.float().contiguous()
    if a2.data_ptr() % 16:  # the GEMM reads activations with 16-byte aligned tensor-memory-access tiles
        a2 = a2.clone()
    M, N = a2.shape[0], b.shape[0]
    as2 = None
    if a_s is not None:
        as2 = a_s.reshape(M, -1).float().contiguous()
        if as2.shape[1] != K // block:
            raise ValueError(f"a_s has {as2.shape[1]} blocks per row, expected {K // block}")
    out_dt = torch.get_default_dtype()
    out = torch.empty((M, N), dtype=torch.float32 if out_dt == torch.float32 else torch.bfloat16, device=a.device)
    _L.call(fn, _L.ptr(a2), adt, _L.ptr(as2), M, K, _L.ptr(_u8(b)), _L.ptr(b_s), N, _L.ptr(out),
            _L.DTYPE_F32 if out.dtype == torch.float32 else _L.DTYPE_BF16, _L.stream_of(a2))
    return out.view(*a.shape[:-1], N).to(out_dt)


def fp8_gemm(a, a_s, b, b_s, scale_dtype=torch.float32, block_size=128):
    """(a * a_s) @ (b * b_s)^T -> default dtype (dsv41/ref/kernel.py:105-107)."""
    if block_size != 128:
        raise NotImplementedError("fp8_gemm supports 128x128 weight blocks")
    return _gemm("dsmoe_fp8_gemm", a, a_s, b, b_s.float().contiguous(), block_size)


def fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32, act_block_size=128):
    """(a * a_s) @ dequant_fp4(b, b_s)^T -> default dtype (dsv41/ref/kernel.py:110-112)."""
    if act_block_size != 128:
        raise NotImplementedError("fp4_gemm supports 128-wide activation blocks")
    return _gemm("dsmoe_fp4_gemm", a, a_s, b, _u8(b_s), act_block_size)


def dequant_fp4_weight(b, b_s):
    """[N, K//2] packed e2m1 (low nibble first) + [N, K//32] e8m0 -> [N, K] float32 (dsv41/ref/kernel.py:91-98)."""
    _cuda(b, b_s)
    N, half = b.shape
    out = torch.empty((N, half * 2), dtype=torch.float32, device=b.device)
    _L.call("dsmoe_fp4_dequant", _L.ptr(_u8(b)), _L.ptr(_u8(b_s)), N, half * 2, _L.ptr(out), _L.DTYPE_F32,
            _L.stream_of(b))
    return out


def weight_dequant(b, b_s, block_size=128):
    """FP8 [N, K] + fp32 (or e8m0) scales per block -> [N, K] in the default dtype."""
    _cuda(b, b_s)
    N, K = b.shape
    out_dt = torch.get_default_dtype()
    out = torch.empty((N, K), dtype=torch.float32 if out_dt == torch.float32 else torch.bfloat16, device=b.device)
    _L.call("dsmoe_fp8_block_dequant", _L.ptr(_u8(b)), _L.ptr(b_s.float().contiguous()), N, K, block_size,
            _L.ptr(out), _L.DTYPE_F32 if out.dtype == torch.float32 else _L.DTYPE_BF16, _L.stream_of(b))
    return out.to(out_dt)


def sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale, chunk=128):
    raise NotImplementedError("sparse attention is outside the MoE expert path this package implements")


def hc_split_sinkhorn(mixes, hc_scale, hc_base, hc_mult=4, sinkhorn_iters=20, eps=1e-6):
    raise NotImplementedError("hyper-connection Sinkhorn is outside the MoE expert path this package implements")
