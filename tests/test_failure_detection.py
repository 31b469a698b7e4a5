"""Failure detection without a GPU fault: a bounded device wait that nothing satisfies must end with
an error status the host reads, and leave the CUDA context usable.

Two processes share one GPU and build a world-2 peer exchange (handles traded over a gloo group).
Rank 1 maps its buffer and then does nothing, so rank 0's waits for rank 1's tiles run out:
- the decode kernel's in-kernel all-reduce (5 s bound) -> a call made before MoE.check returns NaN
  rows at once, MoE.check raises DsmoeError (timeout), and after that reset the layer's own partial
  matches the oracle again;
- the stand-alone row all-reduce (5 s bound) -> PeerComm.check raises DsmoeError (timeout).
Only rank 0 launches kernels, and each wait is bounded by %globaltimer; no kernel waits on another
kernel. This is the device-side counterpart of a collective that never completes because a peer is
gone; nothing here traps, asserts on the device or touches a bad address."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, root, out_q):
    import sys
    for p in (root, os.path.join(root, "tenstorrent-wormhole-deepseek-v41-flash_b200"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120))
    res = {}
    try:
        from dsmoe._lib import DsmoeError
        from dsmoe.tp import PeerComm
        from _util import make_layer_cpu, to_gpu_moe
        comm_decode = PeerComm(1024, device=dev)
        comm_rows = PeerComm(1024, device=dev)
        if rank == 0:
            spec = make_layer_cpu("fp8", 1024, 512, 32, seed=7)
            m = to_gpu_moe(spec, rank=0, world=2, device=dev)
            m.use_comm(comm_decode)
            x = torch.randn((1, 1024), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(dev)
            t0 = time.time()
            m.forward(x)
            torch.cuda.synchronize(dev)
            res["decode_s"] = time.time() - t0
            # a call made before check(): the status word is still set, so it gives up at once and
            # returns NaN rows instead of stale memory
            t0 = time.time()
            y2 = m.forward(x)
            torch.cuda.synchronize(dev)
            res["flagged_nan"] = bool(torch.isnan(y2.float()).all().item())
            res["flagged_s"] = time.time() - t0
            try:
                m.check(1)
                res["decode"] = "no error"
            except DsmoeError as e:
                res["decode"] = "timeout" if "wait expired" in str(e) else repr(e)
            # after check() reset the workspace, the same layer computes correctly again (its fp32
            # partial needs no peer): counters, barrier and tagged router partials were cleared
            import numpy as np
            from oracle import moe as OM
            from _util import to_oracle_layer
            part = m.partial(x).cpu().numpy()
            ref, _, _ = OM.moe_forward(to_oracle_layer(spec), x.float().cpu().numpy(), 0, 2, return_partial=True)
            mar, cos = OM.compare(part, ref)
            res["after_reset"] = bool(mar < 2e-3 and cos > 0.99999 and np.isfinite(part).all())
            m.check(1)
            t0 = time.time()
            comm_rows.allreduce(x)
            try:
                comm_rows.check()
                res["rows"] = "no error"
            except DsmoeError as e:
                res["rows"] = "timeout" if "did not arrive" in str(e) else repr(e)
            res["rows_s"] = time.time() - t0
            # the context still works
            res["alive"] = float(torch.arange(8, device=dev, dtype=torch.float32).sum().item()) == 28.0
        dist.barrier()  # rank 1 keeps its buffers mapped until rank 0 is done
        comm_decode.close()
        comm_rows.close()
        out_q.put((rank, res, None))
    except Exception as ex:  # reported to the parent, which fails the test
        out_q.put((rank, res, repr(ex)))
    finally:
        dist.destroy_process_group()


def test_peer_wait_expires_and_is_reported():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = sorted((q.get(timeout=300) for _ in range(2)), key=lambda t: t[0])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, res, err in got:
        assert err is None, (rank, err)
    res = got[0][1]
    assert res["decode"] == "timeout", res
    assert res["flagged_nan"] and res["flagged_s"] < 4.0, res
    assert res["after_reset"], res
    assert res["rows"] == "timeout", res
    assert 4.0 < res["decode_s"] < 60.0 and 4.0 < res["rows_s"] < 60.0, res
    assert res["alive"], res
    for p in procs:
        assert p.exitcode == 0
