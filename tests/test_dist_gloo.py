"""World-size-2 tensor-parallel host logic on CPU (gloo): each rank computes its slice's partial,
one all-reduce sums them, and the result equals the whole layer; timings reduce to the max."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root, out_q):
    import sys
    for p in (root, os.path.join(root, "tenstorrent-wormhole-deepseek-v41-flash_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from dsmoe.tp import allreduce_partial_, max_over_ranks, slice_of
        from oracle import moe as OM
        from _util import make_layer_cpu, to_oracle_layer
        spec = make_layer_cpu("fp4", 256, 256, 8, seed=31)
        ref = to_oracle_layer(spec)
        x = torch.randn((3, 256), generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).float().numpy()
        row0, loc = slice_of(256, rank, world)
        part, _, _ = OM.moe_forward(ref, x, rank, world, return_partial=True)
        t = torch.from_numpy(part.astype(np.float32))
        allreduce_partial_(t)
        full, _, _ = OM.moe_forward(ref, x, return_partial=True)
        err = float(np.max(np.abs(t.numpy() - full)) / np.max(np.abs(full)))
        slowest = max_over_ranks(1.0 + rank)
        out_q.put((rank, err, slowest, row0, loc))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_allreduce_gloo(world):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, root, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, slowest, row0, loc in res:
        assert err < 1e-6
        assert slowest == float(world)
        assert (row0, loc) == (rank * 256 // world, 256 // world)
