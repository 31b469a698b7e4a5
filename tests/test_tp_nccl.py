"""Tensor parallelism across real GPUs: one process per GPU over NCCL, each rank holding I/world rows
of every expert. Each rank's fused decode writes its fp32 partial, MoE.forward all-reduces them, and
the bf16 result must match the oracle's whole layer on every rank (the all-reduce in
dsv41/tt/attn.py:19-21 sums the same partials). Needs at least two GPUs; skipped otherwise."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

MAR_TOL, COS_TOL = 1e-2, 0.9999


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root, out_q):
    import sys
    for p in (root, os.path.join(root, "tenstorrent-wormhole-deepseek-v41-flash_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    res = []
    try:
        from oracle import moe as OM
        from _util import make_layer_cpu, to_gpu_moe, to_oracle_layer
        for fmt, B in (("fp8", 1), ("fp4", 3), ("fp8", 8), ("fp4", 13)):
            spec = make_layer_cpu(fmt, 1024, 512, 32, seed=4000 + B)
            m = to_gpu_moe(spec, rank=rank, world=world, device=dev)
            x = torch.randn((B, 1024), generator=torch.Generator().manual_seed(B)).to(torch.bfloat16)
            y = m.forward(x.to(dev)).float().cpu().numpy()
            idx, _, _ = m.route(x.to(dev))
            m.check(B)
            yr, ridx, _ = OM.moe_forward(to_oracle_layer(spec), x.float().numpy())
            mar, cos = OM.compare(y, yr)
            res.append((fmt, B, bool(np.array_equal(idx.cpu().numpy(), ridx)), float(mar), float(cos)))
        dist.barrier()
        out_q.put((rank, res, None))
    except Exception as ex:  # reported to the parent, which fails the test
        out_q.put((rank, res, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_forward_nccl(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, root, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = sorted((q.get(timeout=300) for _ in range(world)), key=lambda t: t[0])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, res, err in got:
        assert err is None, (rank, err)
        assert len(res) == 4
        for fmt, B, idx_ok, mar, cos in res:
            assert idx_ok, (rank, fmt, B)
            assert mar < MAR_TOL and cos > COS_TOL, (rank, fmt, B, mar, cos)
    for p in procs:
        assert p.exitcode == 0
