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


def tc_geometry_ok(hidden: int, inter_local: int, n_experts: int, topk: int) -> bool:
    """Shapes the tensor-core decode kernel takes (whole 128-K blocks of hidden up to 8192, at least
    64 intermediate rows per GPU in 32-row steps, up to 1024 experts and top-8)."""
    return (hidden % 128 == 0 and 0 < hidden <= 8192 and 64 <= inter_local <= 8192 and inter_local % 32 == 0
            and n_experts <= 1024 and topk <= 8)


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


def _check_out(out: torch.Tensor, B: int, hidden: int, device) -> None:
    if (out.dtype != torch.bfloat16 or out.shape != (B, hidden) or not out.is_contiguous()
            or out.device != device):
        raise ValueError(f"out must be a contiguous [{B}, {hidden}] bfloat16 tensor on {device}")


class MoE:
    """One MoE layer resident on one GPU (one tensor-parallel rank).

    Build it empty, then load the router, the shared expert and every routed expert from
    checkpoint-layout tensors (they are repacked on the device and may be freed afterwards).
    """

    def __init__(self, hidden: int, inter: int, n_experts: int, topk: int = 6, fmt: str = "fp8",
                 score_func: str = "sigmoid", route_scale: float = 2.5, rank: int = 0, world: int = 1,
                 group=None, device=None, max_tokens: int = L.MAX_DECODE_TOKENS, layouts=("tc", "frag")):
        """``layouts``: the resident stores to keep. "tc" serves decode calls of 1..8 tokens on the
        tensor-core kernel; "frag" serves larger batches and prefill (and decode when "tc" is absent)."""
        if score_func not in L.SCORE_NAMES:
            raise ValueError(f"score_func must be one of {sorted(L.SCORE_NAMES)}")
        layouts = tuple(dict.fromkeys(layouts))
        if not layouts or any(lay not in ("tc", "frag") for lay in layouts):
            raise ValueError("layouts must be a non-empty subset of ('tc', 'frag')")
        loc = inter // world if world > 0 and inter % world == 0 else 0
        if "tc" in layouts and not tc_geometry_ok(hidden, loc, n_experts, topk):
            if layouts == ("tc",):
                raise ValueError(f"the tensor-core store does not take hidden {hidden}, {loc} rows per GPU, "
                                 f"{n_experts} experts, top-{topk}")
            layouts = tuple(lay for lay in layouts if lay != "tc")
        if "frag" in layouts and fmt == "fp4" and loc % 64 and "tc" in layouts:
            layouts = ("tc",)  # the fragment layout keeps FP4 slices in 64-row steps only
        self.hidden, self.inter, self.n_experts, self.topk = hidden, inter, n_experts, topk
        self.fmt, self.score_func, self.route_scale = fmt, score_func, float(route_scale)
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stores = {lay: (ExpertStore(fmt, hidden, inter, n_experts, rank, world, self.device, lay),
                             ExpertStore("fp8", hidden, inter, 1, rank, world, self.device, lay)) for lay in layouts}
        self.routed, self.shared = self.stores["frag" if "frag" in self.stores else "tc"]
        self.wg = torch.zeros((n_experts, hidden), dtype=torch.float32, device=self.device)
        self.bias = torch.zeros((n_experts,), dtype=torch.float32, device=self.device)
        self.bias_vl: Optional[torch.Tensor] = None
        self.max_tokens = min(max_tokens, L.MAX_DECODE_TOKENS)
        self._dec_layout = "tc" if "tc" in self.stores else "frag"
        self._layers = {lay: self._make_layer(lay) for lay in self.stores}
        # workspaces, zero-filled once: the persistent kernels keep counters and tagged partials there
        self._wss = {lay: torch.zeros(L.lib.dsmoe_moe_workspace_bytes(self._layers[lay], self.max_tokens),
                                      dtype=torch.uint8, device=self.device) for lay in self.stores}
        self._bind()
        self.comm = None  # tp.PeerComm: all-reduce inside the decode kernel
        self._prefill_ws: Optional[torch.Tensor] = None  # grown on demand by prefill()

    def use_decode_store(self, layout: str) -> None:
        """Serve decode calls from the given resident store ("tc" or "frag"; it must have been kept)."""
        if layout not in self.stores:
            raise ValueError(f"store {layout!r} is not resident (kept: {tuple(self.stores)})")
        self._dec_layout = layout
        self._bind()

    def _bind(self):
        """The decode layer (tensor-core store when kept) and the batched layer (fragment store)."""
        self._layer = self._layers[self._dec_layout]
        self.workspace = self._wss[self._dec_layout]
        self._ws = (self.workspace.data_ptr(), self.workspace.numel())
        self._dec_max = 8 if self._dec_layout == "tc" else self.max_tokens
        self._layer_b = self._layers.get("frag")
        self.workspace_b = self._wss.get("frag")

    # ---------------------------------------------------------------- loading
    def _make_layer(self, layout: str) -> L.Layer:
        routed, shared = self.stores[layout]
        lay = L.Layer()
        lay.hidden, lay.inter_local, lay.n_experts = self.hidden, routed.inter_local, self.n_experts
        lay.topk, lay.score_func, lay.route_scale = self.topk, L.SCORE_NAMES[self.score_func], self.route_scale
        lay.gate_w, lay.gate_bias = self.wg.data_ptr(), self.bias.data_ptr()
        lay.gate_bias_vl = self.bias_vl.data_ptr() if self.bias_vl is not None else None
        lay.routed, lay.shared = routed.c_struct(), shared.c_struct()
        return lay

    def load_router(self, rw: RouterWeights) -> None:
        self.wg.copy_(rw.wg)
        self.bias.copy_(rw.bias)
        if rw.bias_vl is not None:
            self.bias_vl = rw.bias_vl.to(self.device, torch.float32).contiguous()
        self._layers = {lay: self._make_layer(lay) for lay in self.stores}
        self._bind()

    def load_expert(self, e: int, ew: ExpertWeights) -> None:
        for routed, _ in self.stores.values():
            routed.pack(e, ew)

    def load_shared(self, ew: ExpertWeights) -> None:
        for _, shared in self.stores.values():
            shared.pack(0, ew)

    def copy_experts_from(self, other: "MoE") -> None:
        """Every expert's bytes from a layer of the same geometry (another resident copy)."""
        for lay, (routed, shared) in self.stores.items():
            routed.copy_from(other.stores[lay][0])
            shared.copy_from(other.stores[lay][1])

    @property
    def nbytes(self) -> int:
        return sum(r.nbytes + s.nbytes for r, s in self.stores.values()) + self.wg.numel() * 4 + self.bias.numel() * 4

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
        if self._layer_b is None:
            raise ValueError("prefill reads the fragment store: build the layer with 'frag' in layouts")
        nbytes = L.lib.dsmoe_moe_prefill_workspace_bytes(self._layer_b, P)
        if nbytes == 0:
            raise ValueError(f"prefill does not support this layer with {P} tokens")
        if self._prefill_ws is None or self._prefill_ws.numel() < nbytes:
            self._prefill_ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        f32 = partial or self.world > 1
        y = torch.empty((P, self.hidden), dtype=torch.float32 if f32 else torch.bfloat16, device=self.device)
        L.call("dsmoe_moe_prefill", self._layer_b, L.ptr(x), P, L.ptr(idx), L.ptr(wt), L.ptr(y),
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
            L.call("dsmoe_moe_prefill_check", self._layer_b, P, L.ptr(self._prefill_ws), self._prefill_ws.numel(),
                   L.stream_of(self._prefill_ws))

    def use_comm(self, comm) -> None:
        """Sum the tensor-parallel partials inside the decode kernel over ``comm`` (a tp.PeerComm of
        this layer's group) whenever the call takes the persistent path; None = the collective
        library's all-reduce always."""
        if comm is not None and (comm.world != self.world or comm.rank != self.rank or comm.hidden != self.hidden):
            raise ValueError("comm does not match this layer's rank, world or hidden size")
        self.comm = comm

    def forward(self, x: torch.Tensor, image_mask: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [B, H] bf16: the full layer output (partials all-reduced when world > 1), written into
        ``out`` (a contiguous [B, H] bf16 tensor on the layer's GPU) when given.

        If a bounded device wait of an earlier call on this layer's workspace expired, the kernel
        writes NaN rows instead of y until ``check()`` resets the workspace."""
        if out is not None:
            _check_out(out, x.shape[0], self.hidden, self.device)
        if self.world == 1:
            return self._run(x, image_mask, out, L.DTYPE_BF16)
        if self.comm is not None and self.comm.handle is not None:
            x = _check_x(x, self.hidden, self.device)
            B = x.shape[0]
            if B <= self._dec_max and L.lib.dsmoe_moe_allreduce_supported(self._layer, self.comm.handle,
                                                                           x.data_ptr(), B):
                y = out if out is not None else torch.empty((B, self.hidden), dtype=torch.bfloat16,
                                                            device=self.device)
                mask = self._mask(image_mask, B)
                L.check(L.lib.dsmoe_moe_decode_allreduce(
                    self._layer, self.comm.handle, x.data_ptr(), B, L.ptr(mask), y.data_ptr(), L.DTYPE_BF16, None,
                    None, None, self._ws[0], self._ws[1], torch.cuda.current_stream(self.device).cuda_stream))
                return y
        part = self._run(x, image_mask, None, L.DTYPE_F32)
        torch.distributed.all_reduce(part, group=self.group)
        y = out if out is not None else torch.empty(part.shape, dtype=torch.bfloat16, device=self.device)
        L.call("dsmoe_f32_to_bf16", L.ptr(part), L.ptr(y), part.numel(), L.stream_of(part))
        return y

    __call__ = forward
    decode = forward

    def check(self, B: int = 1) -> None:
        """Synchronize and raise if a bounded device-side wait expired in an earlier call (every
        store's workspace is checked and, after an expired wait, reset)."""
        err = None
        for lay, ws in self._wss.items():
            try:
                L.call("dsmoe_moe_check", self._layers[lay], min(B, self.max_tokens), L.ptr(ws), ws.numel(),
                       L.stream_of(ws))
            except L.DsmoeError as e:
                err = err or e
        if err is not None:
            raise err

    def _run(self, x, image_mask, out, y_dtype, idx=None, wt=None):
        x = _check_x(x, self.hidden, self.device)
        B = x.shape[0]
        if out is None:
            out = torch.empty((B, self.hidden), dtype=torch.float32 if y_dtype == L.DTYPE_F32 else torch.bfloat16,
                              device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        if B <= self._dec_max and image_mask is None and idx is None and wt is None:  # one launch, no slicing
            L.check(L.lib.dsmoe_moe_decode(self._layer, x.data_ptr(), B, None, out.data_ptr(), y_dtype, None, None,
                                           None, self._ws[0], self._ws[1], st))
            return out
        mask = self._mask(image_mask, B)
        # up to 8 tokens on the decode store; larger batches on the fragment store's batched path
        if B <= self._dec_max or self._layer_b is None:
            lay, ws, step = self._layer, self.workspace, self._dec_max
        else:
            lay, ws, step = self._layer_b, self.workspace_b, self.max_tokens
        for b0 in range(0, B, step):
            b1 = min(B, b0 + step)
            L.call("dsmoe_moe_decode", lay, L.ptr(x[b0:b1]), b1 - b0,
                   L.ptr(mask[b0:b1] if mask is not None else None), L.ptr(out[b0:b1]), y_dtype,
                   L.ptr(idx[b0:b1] if idx is not None else None), L.ptr(wt[b0:b1] if wt is not None else None),
                   None, L.ptr(ws), ws.numel(), st)
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
