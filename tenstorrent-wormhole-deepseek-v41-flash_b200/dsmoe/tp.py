"""Tensor-parallel plumbing for the MoE layer (one process per GPU, torch.distributed).

The reference runs the experts TP-8 over its 8-chip mesh: w1/w3 column-parallel, w2 row-parallel,
one all_gather+sum all-reduce of the routed + shared partials per layer (dsv41/tt/moe.py:2-3,
162, 180; dsv41/tt/attn.py:19-21). Here each rank holds a contiguous 1/world slice of every
expert's intermediate dimension and the partials are summed in fp32 with one all-reduce.
"""
import os

import torch


def slice_of(inter: int, rank: int, world: int):
    """(row0, inter_local) of ``rank``'s slice; the slice must keep the packed store's alignment."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if inter % world:
        raise ValueError(f"inter {inter} does not split evenly over {world} ranks")
    loc = inter // world
    if loc % 32:
        raise ValueError(f"per-rank slice {loc} must be a multiple of 32")
    return rank * loc, loc


def allreduce_partial_(part: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the per-rank fp32 partials in place (one all-reduce, as attn.all_reduce_sum does)."""
    if part.dtype != torch.float32:
        raise TypeError("partials are summed in fp32")
    if torch.distributed.is_initialized() and torch.distributed.get_world_size(group) > 1:
        torch.distributed.all_reduce(part, op=torch.distributed.ReduceOp.SUM, group=group)
    return part


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The slowest rank's value (benchmark times are the max over ranks)."""
    if not (torch.distributed.is_initialized() and torch.distributed.get_world_size(group) > 1):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
    return float(t.item())


def env_rank_world():
    """(rank, local_rank, world) from torchrun's environment (1 process when absent)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


class PeerComm:
    """One rank's end of the all-reduce inside the decode kernel (``dsmoe_comm`` of libdsmoe.so).

    An exchange buffer on this GPU that every other rank of ``group`` maps with CUDA IPC; a layer
    called through it (``MoE.forward`` once ``MoE.use_comm`` is set) stores its output tiles into the
    peers' buffers over NVLink and sums what it receives, in one launch per rank -- the role of the
    reference's ``all_reduce_sum`` after each MoE layer (dsv41/tt/attn.py:19-21). Collective: every
    rank of ``group`` constructs it, with its own GPU current. One comm serves any number of layers
    of the same hidden size, provided every rank calls them in the same order.
    """

    def __init__(self, hidden: int, group=None, device=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib as L
        self.rank, self.world, self.hidden = dist.get_rank(group), dist.get_world_size(group), hidden
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        handle = (ctypes.c_uint8 * L.COMM_HANDLE_BYTES)()
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.call("dsmoe_comm_create", self.rank, self.world, hidden, ctypes.byref(p), handle)
            self.handle = p.value
            try:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
                L.call("dsmoe_comm_open", self.handle, b"".join(handles))
            except Exception:
                L.lib.dsmoe_comm_destroy(self.handle)
                self.handle = None
                raise

    def allreduce(self, x: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
        """Sum [B, hidden] (B <= 8, bf16 or fp32) over the group through the peer exchange, in one
        launch (the reference's all_reduce_sum after the attention output projection,
        dsv41/tt/attn.py:19-21). Every rank gets the same bits; rows beyond 8 go in several calls."""
        from . import _lib as L
        if x.dim() != 2 or x.shape[1] != self.hidden or x.device != self.device:
            raise ValueError(f"x must be [rows, {self.hidden}] on {self.device}")
        dt = {torch.bfloat16: L.DTYPE_BF16, torch.float32: L.DTYPE_F32}.get(x.dtype)
        if dt is None:
            raise TypeError("x must be bfloat16 or float32")
        x = x.contiguous()
        y = torch.empty_like(x) if out is None else out
        for r0 in range(0, x.shape[0], 8):
            r1 = min(x.shape[0], r0 + 8)
            L.call("dsmoe_allreduce_rows", self.handle, L.ptr(x[r0:r1]), dt, r1 - r0, L.ptr(y[r0:r1]), dt,
                   L.stream_of(x))
        return y

    def check(self) -> None:
        """Synchronize and raise if a peer's tile did not arrive in time in allreduce()."""
        from . import _lib as L
        L.call("dsmoe_comm_check", self.handle, L.stream_of())

    def close(self) -> None:
        """Free this rank's buffer and unmap the peers' (synchronizes the device)."""
        from . import _lib as L
        if self.handle is not None:
            with torch.cuda.device(self.device):
                L.call("dsmoe_comm_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
