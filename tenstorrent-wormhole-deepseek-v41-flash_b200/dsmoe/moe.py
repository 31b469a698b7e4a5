"""MoE layer host classes: Gate, Expert, MoE -- the reference's operator surface over the CUDA path.

Reference surface mirrored:
* DeepSeek model.py ``Gate.forward(x, image_mask=None) -> (weights, indices)`` (as wrapped by
  dsv41/ref/load.py:70-79) and the engine's ``MoE.route(x, image_mask) -> (idx, wt, sc)``
  (dsv41/tt/moe.py:114-125);
* ``Expert`` forward (dsv41/tt/moe.py:133-139 ``_ffn``);
* ``MoE.forward`` / ``MoE.decode`` (dsv41/tt/moe.py:148-180, 202-241): routed + shared experts,
  routing weight applied before w2, one all-reduce of the partial sums over the tensor-parallel
  group (dsv41/tt/attn.py:19-21).

Everything runs on the GPU through libdsmoe.so; there is no CPU path. Tensors are row-major
``[tokens, hidden]`` bf16, weights ``[out, in]`` as in the checkpoint.
"""
from typing import Optional

import torch

from . import _lib as L
from .store import ExpertStore
from .synth import ExpertWeights, RouterWeights

LIMIT = 10.0  # SwiGLU clamp (dsv41/tt/moe.py:15)


def _check_x(x: torch.Tensor, hidden: int, device) -> torch.Tensor:
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != hidden or x.device != device:
        if not x.is_cuda:
            raise ValueError("dsmoe runs on CUDA tensors only")
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        if x.dim() != 2 or x.shape[1] != hidden:
            raise ValueError(f"x must be [tokens, {hidden}], got {tuple(x.shape)}")
        raise ValueError(f"x is on {x.device}, layer on {device}")
    return x if x.is_contiguous() else x.contiguous()


class MoE:
    """One MoE layer resident on one GPU (one tensor-parallel rank).

    Build it empty, then load the router, the shared expert and every routed expert from
    checkpoint-layout tensors (they are repacked on the device and may be freed afterwards).
    """

    def __init__(self, hidden: int, inter: int, n_experts: int, topk: int = 6, fmt: str = "fp8",
                 score_func: str = "sigmoid", route_scale: float = 2.5, rank: int = 0, world: int = 1,
                 group=None, device=None, max_tokens: int = L.MAX_DECODE_TOKENS):
        if score_func not in L.SCORE_NAMES:
            raise ValueError(f"score_func must be one of {sorted(L.SCORE_NAMES)}")
        self.hidden, self.inter, self.n_experts, self.topk = hidden, inter, n_experts, topk
        self.fmt, self.score_func, self.route_scale = fmt, score_func, float(route_scale)
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.routed = ExpertStore(fmt, hidden, inter, n_experts, rank, world, self.device)
        self.shared = ExpertStore("fp8", hidden, inter, 1, rank, world, self.device)
        self.wg = torch.zeros((n_experts, hidden), dtype=torch.float32, device=self.device)
        self.bias = torch.zeros((n_experts,), dtype=torch.float32, device=self.device)
        self.bias_vl: Optional[torch.Tensor] = None
        self.max_tokens = min(max_tokens, L.MAX_DECODE_TOKENS)
        self._layer = self._make_layer()
        nbytes = L.lib.dsmoe_moe_workspace_bytes(self._layer, self.max_tokens)
        # zero-filled once: the persistent kernel keeps counters and a grid barrier here
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self._ws = (self.workspace.data_ptr(), self.workspace.numel())
        self.comm = None  # tp.PeerComm: all-reduce inside the decode kernel
        self._prefill_ws: Optional[torch.Tensor] = None  # grown on demand by prefill()

    # ---------------------------------------------------------------- loading
    def _make_layer(self) -> L.Layer:
        lay = L.Layer()
        lay.hidden, lay.inter_local, lay.n_experts = self.hidden, self.routed.inter_local, self.n_experts
        lay.topk, lay.score_func, lay.route_scale = self.topk, L.SCORE_NAMES[self.score_func], self.route_scale
        lay.gate_w, lay.gate_bias = self.wg.data_ptr(), self.bias.data_ptr()
        lay.gate_bias_vl = self.bias_vl.data_ptr() if self.bias_vl is not None else None
        lay.routed, lay.shared = self.routed.c_struct(), self.shared.c_struct()
        return lay

    def load_router(self, rw: RouterWeights) -> None:
        self.wg.copy_(rw.wg)
        self.bias.copy_(rw.bias)
        if rw.bias_vl is not None:
            self.bias_vl = rw.bias_vl.to(self.device, torch.float32).contiguous()
        self._layer = self._make_layer()

    def load_expert(self, e: int, ew: ExpertWeights) -> None:
        self.routed.pack(e, ew)

    def load_shared(self, ew: ExpertWeights) -> None:
        self.shared.pack(0, ew)

    @property
    def nbytes(self) -> int:
        return self.routed.nbytes + self.shared.nbytes + self.wg.numel() * 4 + self.bias.numel() * 4

    # ---------------------------------------------------------------- router
    def route(self, x: torch.Tensor, image_mask: Optional[torch.Tensor] = None):
        """(idx [B, k] int64, wt [B, k] fp32, sc [B, E] fp32), all on the GPU (dsv41/tt/moe.py:114-125)."""
        x = _check_x(x, self.hidden, self.device)
        B = x.shape[0]
        idx = torch.empty((B, self.topk), dtype=torch.int64, device=self.device)
        wt = torch.empty((B, self.topk), dtype=torch.float32, device=self.device)
        sc = torch.empty((B, self.n_experts), dtype=torch.float32, device=self.device)
        mask = self._mask(image_mask, B)
        for b0 in range(0, B, self.max_tokens):
            b1 = min(B, b0 + self.max_tokens)
            L.call("dsmoe_router", self._layer, L.ptr(x[b0:b1]), b1 - b0, L.ptr(mask[b0:b1] if mask is not None else None),
                   L.ptr(idx[b0:b1]), L.ptr(wt[b0:b1]), L.ptr(sc[b0:b1]), L.ptr(self.workspace),
                   self.workspace.numel(), L.stream_of(x))
        return idx, wt, sc

    def _mask(self, image_mask, B):
        if image_mask is None:
            return None
        m = image_mask.to(self.device, torch.uint8).contiguous()
        if m.shape != (B,):
            raise ValueError("image_mask must be [tokens]")
        return m

    # ---------------------------------------------------------------- forward
    def partial(self, x: torch.Tensor, image_mask: Optional[torch.Tensor] = None, out=None,
                idx=None, wt=None) -> torch.Tensor:
        """This rank's fp32 partial sum [B, H] (routed + shared over its intermediate slice)."""
        return self._run(x, image_mask, out, L.DTYPE_F32, idx, wt)

    def prefill(self, x: torch.Tensor, idx: Optional[torch.Tensor] = None, wt: Optional[torch.Tensor] = None,
                image_mask: Optional[torch.Tensor] = None, partial: bool = False) -> torch.Tensor:
        """Batched layer for P tokens on the tcgen05 grouped GEMMs (dsv41/tt/moe.py:182-200, 263-288).

        Routing comes from ``idx`` [P, k] int64 / ``wt`` [P, k] fp32 when given (e.g. forced), else
        from this layer's router. Returns y [P, H] bf16 -- all-reduced over the tensor-parallel group
        when world > 1 -- or this rank's fp32 partial with ``partial=True``."""
        x = _check_x(x, self.hidden, self.device)
        P = x.shape[0]
        if idx is None:
            idx, wt, _ = self.route(x, image_mask)
        elif wt is None:
            raise ValueError("wt is required with idx")
        idx = idx.to(self.device, torch.int64).contiguous()
        wt = wt.to(self.device, torch.float32).contiguous()
        if idx.shape != (P, self.topk) or wt.shape != (P, self.topk):
            raise ValueError(f"idx / wt must be [{P}, {self.topk}]")
        nbytes = L.lib.dsmoe_moe_prefill_workspace_bytes(self._layer, P)
        if nbytes == 0:
            raise ValueError(f"prefill does not support this layer with {P} tokens")
        if self._prefill_ws is None or self._prefill_ws.numel() < nbytes:
            self._prefill_ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        f32 = partial or self.world > 1
        y = torch.empty((P, self.hidden), dtype=torch.float32 if f32 else torch.bfloat16, device=self.device)
        L.call("dsmoe_moe_prefill", self._layer, L.ptr(x), P, L.ptr(idx), L.ptr(wt), L.ptr(y),
               L.DTYPE_F32 if f32 else L.DTYPE_BF16, L.ptr(self._prefill_ws), self._prefill_ws.numel(), L.stream_of(x))
        if partial or self.world == 1:
            return y
        torch.distributed.all_reduce(y, group=self.group)
        out = torch.empty((P, self.hidden), dtype=torch.bfloat16, device=self.device)
        L.call("dsmoe_f32_to_bf16", L.ptr(y), L.ptr(out), y.numel(), L.stream_of(y))
        return out

    def prefill_check(self, P: int) -> None:
        """Synchronize and raise if the last prefill call's bounded waits expired or an index was bad."""
        if self._prefill_ws is not None:
            L.call("dsmoe_moe_prefill_check", self._layer, P, L.ptr(self._prefill_ws), self._prefill_ws.numel(),
                   L.stream_of(self._prefill_ws))

    def use_comm(self, comm) -> None:
        """Sum the tensor-parallel partials inside the decode kernel over ``comm`` (a tp.PeerComm of
        this layer's group) whenever the call takes the persistent path; None = the collective
        library's all-reduce always."""
        if comm is not None and (comm.world != self.world or comm.rank != self.rank or comm.hidden != self.hidden):
            raise ValueError("comm does not match this layer's rank, world or hidden size")
        self.comm = comm

    def forward(self, x: torch.Tensor, image_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [B, H] bf16: the full layer output (partials all-reduced when world > 1).

        If a bounded device wait of an earlier call on this layer's workspace expired, the kernel
        writes NaN rows instead of y until ``check()`` resets the workspace."""
        if self.world == 1:
            return self._run(x, image_mask, None, L.DTYPE_BF16)
        if self.comm is not None and self.comm.handle is not None:
            x = _check_x(x, self.hidden, self.device)
            B = x.shape[0]
            if B <= self.max_tokens and L.lib.dsmoe_moe_allreduce_supported(self._layer, self.comm.handle,
                                                                             x.data_ptr(), B):
                y = torch.empty((B, self.hidden), dtype=torch.bfloat16, device=self.device)
                mask = self._mask(image_mask, B)
                L.check(L.lib.dsmoe_moe_decode_allreduce(
                    self._layer, self.comm.handle, x.data_ptr(), B, L.ptr(mask), y.data_ptr(), L.DTYPE_BF16, None,
                    None, None, self._ws[0], self._ws[1], torch.cuda.current_stream(self.device).cuda_stream))
                return y
        part = self._run(x, image_mask, None, L.DTYPE_F32)
        torch.distributed.all_reduce(part, group=self.group)
        y = torch.empty(part.shape, dtype=torch.bfloat16, device=self.device)
        L.call("dsmoe_f32_to_bf16", L.ptr(part), L.ptr(y), part.numel(), L.stream_of(part))
        return y

    __call__ = forward
    decode = forward

    def check(self, B: int = 1) -> None:
        """Synchronize and raise if a bounded device-side wait expired in an earlier call."""
        L.call("dsmoe_moe_check", self._layer, min(B, self.max_tokens), L.ptr(self.workspace),
               self.workspace.numel(), L.stream_of(self.workspace))

    def _run(self, x, image_mask, out, y_dtype, idx=None, wt=None):
        x = _check_x(x, self.hidden, self.device)
        B = x.shape[0]
        if out is None:
            out = torch.empty((B, self.hidden), dtype=torch.float32 if y_dtype == L.DTYPE_F32 else torch.bfloat16,
                              device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        if B <= self.max_tokens and image_mask is None and idx is None and wt is None:  # one launch, no slicing
            L.check(L.lib.dsmoe_moe_decode(self._layer, x.data_ptr(), B, None, out.data_ptr(), y_dtype, None, None,
                                           None, self._ws[0], self._ws[1], st))
            return out
        mask = self._mask(image_mask, B)
        for b0 in range(0, B, self.max_tokens):
            b1 = min(B, b0 + self.max_tokens)
            L.call("dsmoe_moe_decode", self._layer, L.ptr(x[b0:b1]), b1 - b0,
                   L.ptr(mask[b0:b1] if mask is not None else None), L.ptr(out[b0:b1]), y_dtype,
                   L.ptr(idx[b0:b1] if idx is not None else None), L.ptr(wt[b0:b1] if wt is not None else None),
                   None, L.ptr(self.workspace), self.workspace.numel(), st)
        return out


class Gate:
    """DeepSeek-style gate over a MoE layer's router: forward(x) -> (weights [B,k], indices [B,k])."""

    def __init__(self, moe: MoE):
        self.moe = moe

    def forward(self, x: torch.Tensor, image_mask: Optional[torch.Tensor] = None):
        idx, wt, _ = self.moe.route(x, image_mask)
        return wt, idx

    __call__ = forward


class Expert:
    """One expert FFN on checkpoint-layout weights through the kernel-surface GEMMs.

    y = w2( (silu(min(w1 x, 10)) * clamp(w3 x, -10, 10)) * weight ), fp32 intermediates
    (dsv41/tt/moe.py:133-139). Useful outside the fused decode path (tests, one-off calls).
    """

    def __init__(self, ew: ExpertWeights, device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ew = ew.to(dev)
        self.device = dev

    def _lin(self, a: torch.Tensor, q, s, n_out: int) -> torch.Tensor:
        a = a.contiguous()
        out = torch.empty((a.shape[0], n_out), dtype=torch.float32, device=self.device)
        fn = "dsmoe_fp8_gemm" if self.ew.fmt == "fp8" else "dsmoe_fp4_gemm"
        L.call(fn, L.ptr(a), L.DTYPE_F32 if a.dtype == torch.float32 else L.DTYPE_BF16, None, a.shape[0], a.shape[1],
               L.ptr(q), L.ptr(s), n_out, L.ptr(out), L.DTYPE_F32, L.stream_of(a))
        return out

    def forward(self, x: torch.Tensor, weight: Optional[torch.Tensor] = None) -> torch.Tensor:
        inter, hidden = self.ew.w1.shape[0], x.shape[1]
        g = self._lin(x, self.ew.w1, self.ew.s1, inter).clamp(max=LIMIT)
        u = self._lin(x, self.ew.w3, self.ew.s3, inter).clamp(min=-LIMIT, max=LIMIT)
        h = torch.nn.functional.silu(g) * u
        if weight is not None:
            h = h * weight.float().view(-1, 1)
        return self._lin(h, self.ew.w2, self.ew.s2, hidden)

    __call__ = forward
