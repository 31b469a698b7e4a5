"""The tensor-core decode path (tcgen05 + TMA tensor maps on the checkpoint-order store) against the
oracle, through the C ABI.

Bars as for every layer test: router indices bit-exact, bf16 outputs within max-abs-rel 1e-2 and
cosine 0.9999 of the fp32-dequant reference, fp32 partials within 2e-3 / 0.99999; the store
itself bit-exact (its scale tables are what the kernel reads)."""
import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import moe as OM

from _util import bf16_np, make_layer_cpu, to_gpu_moe, to_oracle_layer

pytestmark = pytest.mark.gpu

MAR_TOL, COS_TOL = 1e-2, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401
    return torch.device("cuda", 0)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("inter,world,rank", [(512, 1, 0), (512, 2, 1), (512, 8, 5), (2304, 8, 3), (2304, 8, 7)])
def test_tc_store_bit_exact(dev, fmt, inter, world, rank):
    """Unpack of the tensor-core store == the reference dequant of the rank's slice, bit for bit
    (at 2304 / 8 = 288 rows per rank, FP8 row blocks and w2 K blocks straddle the slice)."""
    from dsmoe import ExpertStore, synth
    H = 512
    gen = torch.Generator().manual_seed(inter + rank)
    ew = synth.make_expert(fmt, H, inter, gen)
    deq = F.dequant_fp8_block if fmt == "fp8" else F.dequant_fp4
    full = {n: deq(getattr(ew, n).numpy(), getattr(ew, "s" + n[1:]).numpy()) for n in ("w1", "w3", "w2")}
    st = ExpertStore(fmt, H, inter, 2, rank, world, dev, layout="tc")
    st.pack(1, ew)
    w1, w3, w2 = (t.cpu().numpy() for t in st.unpack(1))
    loc = inter // world
    sl = slice(rank * loc, (rank + 1) * loc)
    assert np.array_equal(bits(w1), bits(full["w1"][sl]))
    assert np.array_equal(bits(w3), bits(full["w3"][sl]))
    assert np.array_equal(bits(w2), bits(full["w2"][:, sl]))


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("B", [1, 2, 5, 8])
def test_tc_layer_vs_oracle(dev, fmt, B):
    spec = make_layer_cpu(fmt, 1024, 512, 32, seed=5000 + B)
    m = to_gpu_moe(spec, device=dev)
    assert m._dec_layout == "tc"
    ref = to_oracle_layer(spec)
    x = torch.randn((B, 1024), generator=torch.Generator().manual_seed(70 + B)).to(torch.bfloat16)
    y = bf16_np(m.forward(x.to(dev)))
    part = m.partial(x.to(dev)).cpu().numpy()
    idx, _, _ = m.route(x.to(dev))
    m.check(B)
    yr, ridx, _ = OM.moe_forward(ref, x.float().numpy())
    assert np.array_equal(idx.cpu().numpy(), ridx)
    mar, cos = OM.compare(y, yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
    yp, _, _ = OM.moe_forward(ref, x.float().numpy(), return_partial=True)
    mar32, cos32 = OM.compare(part, yp)
    assert mar32 < 2e-3 and cos32 > 0.99999, (mar32, cos32)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("inter,world", [(512, 2), (512, 8), (2304, 8)])
def test_tc_tp_partials(dev, fmt, inter, world):
    """Every rank's slice built side by side on one GPU: partials match the oracle's, and sum to the
    layer (at 2304 / 8 the real model's 288-row slices, FP4 included)."""
    spec = make_layer_cpu(fmt, 512, inter, 16, seed=inter + world)
    ref = to_oracle_layer(spec)
    x = torch.randn((3, 512), generator=torch.Generator().manual_seed(world)).to(torch.bfloat16)
    tot = None
    for r in range(world):
        m = to_gpu_moe(spec, rank=r, world=world, device=dev)
        assert m._dec_layout == "tc"
        p = m.partial(x.to(dev)).cpu().numpy().astype(np.float64)
        m.check(3)
        pr, _, _ = OM.moe_forward(ref, x.float().numpy(), r, world, return_partial=True)
        mar, cos = OM.compare(p, pr)
        assert mar < 2e-3 and cos > 0.99999, (r, mar, cos)
        tot = p if tot is None else tot + p
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    mar, cos = OM.compare(F.bf16_round(tot.astype(np.float32)), yr)
    assert mar < MAR_TOL and cos > COS_TOL


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_tc_many_calls_and_graph(dev, fmt):
    """One workspace, many calls of varying batch (launch-tagged counters never reset), then the same
    call captured in a CUDA graph and replayed: every output equals the first one bit for bit."""
    spec = make_layer_cpu(fmt, 1024, 256, 32, seed=91)
    m = to_gpu_moe(spec, device=dev)
    gen = torch.Generator().manual_seed(92)
    xs = [torch.randn((B, 1024), generator=gen).to(torch.bfloat16).to(dev) for B in (1, 8, 3, 1, 6)]
    first = [m.forward(x).clone() for x in xs]
    for it in range(20):
        j = it % len(xs)
        assert torch.equal(m.forward(xs[j]), first[j]), it
    m.check(8)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        m.forward(xs[0])
    torch.cuda.current_stream(dev).wait_stream(st)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = m.forward(xs[0])
    for _ in range(5):
        g.replay()
        torch.cuda.synchronize(dev)
        assert torch.equal(yg, first[0])
    del g
    m.check(1)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("B", [1, 8])
def test_fragment_path_still_serves(dev, fmt, B):
    """The fragment-layout persistent kernel (kept for layers built without the tensor-core store)."""
    spec = make_layer_cpu(fmt, 1024, 512, 32, seed=6000 + B)
    from dsmoe import MoE
    m = MoE(1024, 512, 32, 6, fmt, device=dev, layouts=("frag",))
    m.load_router(spec["router"])
    m.load_shared(spec["shared"])
    for e, ew in enumerate(spec["experts"]):
        m.load_expert(e, ew)
    x = torch.randn((B, 1024), generator=torch.Generator().manual_seed(B)).to(torch.bfloat16)
    y = bf16_np(m.forward(x.to(dev)))
    m.check(B)
    yr, _, _ = OM.moe_forward(to_oracle_layer(spec), x.float().numpy())
    mar, cos = OM.compare(y, yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
