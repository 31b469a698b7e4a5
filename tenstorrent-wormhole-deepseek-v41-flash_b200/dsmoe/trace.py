"""Traced decode: the decode calls of a fixed set of MoE layers captured once as a CUDA graph and
replayed every step.

This is the B200 counterpart of the reference's ``DecodeTrace`` (dsv41/tt/model.py:262-330), which
captures the per-token device work once and replays it, with every per-token input at a fixed
address and every output written into buffers allocated before the capture. Here the graph holds,
in order: one copy (``dsmoe_copy_async``, a memcpy node) of the step's tokens from pinned host
memory into the device input buffer, one decode launch per layer (each writing its rows of one
device output buffer), and one copy of all outputs back to pinned host memory. A step is then one graph launch and one synchronize, with no
per-layer Python or driver work.

Rules (the same as the reference's trace):
- the layers, their token count and, at world > 1, their comm are fixed at construction; a layer
  whose weights are reloaded keeps its buffers, so the trace stays valid;
- at world > 1 the layers sum their partials inside the decode kernel (a PeerComm attached, at
  most 8 tokens), so the graph holds no collective-library call; every rank builds its trace over
  the same layers in the same order (the warm-up calls run the exchange) and replays it in step
  with the other ranks;
- a bounded device wait that expires inside a replay leaves NaN rows in the outputs, and
  ``check()`` (every layer's ``MoE.check``) reports it.
"""
from typing import Optional, Sequence

import torch

from . import _lib as L
from .moe import MoE


class DecodeTrace:
    """``layers[i]`` decodes ``x_host[i]`` ([tokens, hidden] bf16) into ``y_host[i]`` every step.

    >>> tr = DecodeTrace([moe_a, moe_b], tokens=1)
    >>> tr.x_host.copy_(x)        # or tr.step(x)
    >>> tr.step()                 # y in tr.y_host, already synchronized
    """

    WARM = 2  # eager calls before the capture: every lazily created resource exists by then

    def __init__(self, layers: Sequence[MoE], tokens: int):
        layers = list(layers)
        if not layers:
            raise ValueError("DecodeTrace needs at least one layer")
        dev, H = layers[0].device, layers[0].hidden
        for m in layers:
            if m.device != dev or m.hidden != H:
                raise ValueError("every layer of a trace must share one GPU and one hidden size")
        if not 1 <= tokens <= min(m.max_tokens for m in layers):
            raise ValueError(f"tokens must be in [1, {min(m.max_tokens for m in layers)}]")
        for m in layers:
            if m.world > 1 and (m.comm is None or tokens > 8):
                raise ValueError("at world > 1 a trace replays the in-kernel all-reduce: attach a PeerComm "
                                 "(MoE.use_comm) and trace at most 8 tokens")
        self.layers, self.tokens, self.device = layers, tokens, dev
        n = len(layers)
        self.x_host = torch.zeros((n, tokens, H), dtype=torch.bfloat16).pin_memory()
        self.y_host = torch.zeros((n, tokens, H), dtype=torch.bfloat16).pin_memory()
        self._xd = torch.zeros((n, tokens, H), dtype=torch.bfloat16, device=dev)
        self._yd = torch.zeros((n, tokens, H), dtype=torch.bfloat16, device=dev)
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(self.WARM):
                self._body()
        cur.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        torch.cuda.synchronize(dev)

    def _body(self) -> None:
        st = L.stream_of(self._xd)
        L.call("dsmoe_copy_async", self._xd.data_ptr(), self.x_host.data_ptr(), self.h2d_bytes, st)
        for i, m in enumerate(self.layers):
            m.forward(self._xd[i], out=self._yd[i])
        L.call("dsmoe_copy_async", self.y_host.data_ptr(), self._yd.data_ptr(), self.d2h_bytes, st)

    @property
    def h2d_bytes(self) -> int:
        return self.x_host.numel() * self.x_host.element_size()

    @property
    def d2h_bytes(self) -> int:
        return self.y_host.numel() * self.y_host.element_size()

    def step(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One traced decode step. ``x`` ([layers, tokens, hidden] bf16 on the host), when given, is
        copied into ``x_host`` first. Returns ``y_host`` after the step's copies have landed."""
        if self.graph is None:
            raise RuntimeError("this DecodeTrace was released")
        if x is not None:
            self.x_host.copy_(x)
        self.graph.replay()
        torch.cuda.current_stream(self.device).synchronize()
        return self.y_host

    def check(self) -> None:
        """Raise if a bounded device wait expired in any layer since the last check."""
        for m in self.layers:
            m.check(self.tokens)

    def release(self) -> None:
        """Free the graph (before the process group of the layers' comm is destroyed)."""
        self.graph = None
