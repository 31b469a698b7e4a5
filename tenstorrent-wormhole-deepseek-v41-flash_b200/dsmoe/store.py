"""Resident expert store for one MoE layer on one GPU.

Replaces the reference's host expert store and slot pool (dsv41/tt/store.py:15-120 -- per-(layer,
expert, proj) files packed on demand -- and ExpertPool / Slots, dsv41/tt/moe.py:36-94 -- six device
slots per layer, paged in with host-to-device copies on a miss). Here every expert of the layer is
repacked once on the device into the packed fragment-order layout (csrc/store.cu) and stays
resident; the decode kernels index it by expert id, so nothing is paged or gathered per token.
Two layouts exist: the fragment-order tiles of the legacy kernels (csrc/store.cu) and the tensor-core
layout (csrc/tcstore.cuh) -- checkpoint row-major weights that TMA tensor maps tile on the fly.

With tensor parallelism over ``world`` GPUs, rank r keeps rows [r*I/world, (r+1)*I/world) of every
expert's intermediate dimension (w1/w3 column-parallel, w2 row-parallel; dsv41/tt/moe.py:2-3).
"""
import ctypes

import torch

from . import _lib as L
from .synth import ExpertWeights


def expert_bytes(fmt: str, hidden: int, inter_local: int, layout: str = "frag", inter: int = None, row0: int = 0):
    a, b = ctypes.c_longlong(), ctypes.c_longlong()
    if layout == "tc":
        L.call("dsmoe_store_tc_expert_bytes", L.FMT_NAMES[fmt], hidden, inter if inter is not None else row0 + inter_local,
               row0, inter_local, ctypes.byref(a), ctypes.byref(b))
    else:
        L.call("dsmoe_store_expert_bytes", L.FMT_NAMES[fmt], hidden, inter_local, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


LAYOUTS = {"frag": L.LAYOUT_FRAG, "tc": L.LAYOUT_TC}


def _aligned_empty(nbytes: int, device, align: int = 1024) -> torch.Tensor:
    """Uninitialised bytes whose first address is a multiple of ``align`` (TMA tensor maps)."""
    buf = torch.empty(nbytes + align, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % align
    return buf[off:off + nbytes]


class ExpertStore:
    """``layout`` "frag": packed fragment-order tiles read by the legacy decode kernels and the
    prefill path; "tc": the checkpoint's row-major order plus per-tile scale tables, read by the
    tensor-core decode kernel through TMA tensor maps."""

    def __init__(self, fmt: str, hidden: int, inter: int, n_experts: int, rank: int = 0, world: int = 1,
                 device=None, layout: str = "frag"):
        if fmt not in L.FMT_NAMES:
            raise ValueError(f"unknown format {fmt!r}")
        if layout not in LAYOUTS:
            raise ValueError(f"unknown layout {layout!r}")
        if inter % world:
            raise ValueError(f"inter {inter} does not split over {world} ranks")
        self.fmt, self.hidden, self.inter, self.n_experts = fmt, hidden, inter, n_experts
        self.rank, self.world, self.layout = rank, world, layout
        self.inter_local = inter // world
        self.row0 = rank * self.inter_local
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.w13_expert_bytes, self.w2_expert_bytes = expert_bytes(fmt, hidden, self.inter_local, layout, inter,
                                                                   self.row0)
        self.w13 = _aligned_empty(n_experts * self.w13_expert_bytes, self.device)
        self.w2 = _aligned_empty(n_experts * self.w2_expert_bytes, self.device)

    @property
    def nbytes(self) -> int:
        return self.w13.numel() + self.w2.numel()

    def _w13(self, e):
        return self.w13[e * self.w13_expert_bytes:(e + 1) * self.w13_expert_bytes]

    def _w2(self, e):
        return self.w2[e * self.w2_expert_bytes:(e + 1) * self.w2_expert_bytes]

    def pack(self, e: int, ew: ExpertWeights) -> None:
        """Repack expert ``e`` from checkpoint layout (any device; copied to this GPU if needed)."""
        if ew.fmt != self.fmt:
            raise ValueError(f"expert format {ew.fmt} != store format {self.fmt}")
        if not 0 <= e < self.n_experts:
            raise IndexError(e)
        t = [getattr(ew, n).to(self.device).contiguous() for n in ("w1", "s1", "w3", "s3", "w2", "s2")]
        kh = self.hidden if self.fmt == "fp8" else self.hidden // 2
        ki = self.inter if self.fmt == "fp8" else self.inter // 2
        if tuple(t[0].shape) != (self.inter, kh) or tuple(t[4].shape) != (self.hidden, ki):
            raise ValueError(f"expert shapes {tuple(t[0].shape)}, {tuple(t[4].shape)} do not match "
                             f"hidden {self.hidden} / inter {self.inter} ({self.fmt})")
        fn = "dsmoe_store_tc_pack_expert" if self.layout == "tc" else "dsmoe_store_pack_expert"
        with torch.cuda.device(self.device):
            L.call(fn, L.FMT_NAMES[self.fmt], self.hidden, self.inter, self.row0, self.inter_local,
                   *(L.ptr(x) for x in t), L.ptr(self._w13(e)), L.ptr(self._w2(e)), L.stream_of(self.w13))

    def unpack(self, e: int):
        """Expert ``e``'s slice back in checkpoint layout, dequantized to fp32: (w1, w3 [I_loc, H], w2 [H, I_loc])."""
        w1 = torch.empty((self.inter_local, self.hidden), dtype=torch.float32, device=self.device)
        w3 = torch.empty_like(w1)
        w2 = torch.empty((self.hidden, self.inter_local), dtype=torch.float32, device=self.device)
        fn = "dsmoe_store_tc_unpack_expert" if self.layout == "tc" else "dsmoe_store_unpack_expert"
        with torch.cuda.device(self.device):
            L.call(fn, L.FMT_NAMES[self.fmt], self.hidden, self.inter, self.row0, self.inter_local,
                   L.ptr(self._w13(e)), L.ptr(self._w2(e)), L.ptr(w1), L.ptr(w3), L.ptr(w2), L.stream_of(self.w13))
        return w1, w3, w2

    def copy_from(self, other: "ExpertStore") -> None:
        """Bytes of a store of the same geometry and layout (a second resident copy)."""
        if (other.fmt, other.hidden, other.inter, other.n_experts, other.rank, other.world, other.layout) != \
                (self.fmt, self.hidden, self.inter, self.n_experts, self.rank, self.world, self.layout):
            raise ValueError("store geometry differs")
        self.w13.copy_(other.w13)
        self.w2.copy_(other.w2)

    def c_struct(self) -> L.Store:
        return L.Store(self.w13.data_ptr(), self.w2.data_ptr(), self.w13_expert_bytes, self.w2_expert_bytes,
                       L.FMT_NAMES[self.fmt], self.n_experts, LAYOUTS[self.layout], self.row0)
