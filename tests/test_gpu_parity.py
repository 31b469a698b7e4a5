"""CUDA path vs the oracle (and vs the reference's golden vectors), through the C ABI.

Bars (from the benchmark's north star): router indices and weight unpacking bit-exact; bf16
layer outputs within max-abs-rel 1e-2 and cosine >= 0.9999 of the fp32-dequant reference.
"""
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
    import dsmoe  # noqa: F401  (fails loudly if libdsmoe.so is missing)
    return torch.device("cuda", 0)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


# ------------------------------------------------------------------ unpack (bit-exact)

def test_fp4_dequant_golden(dev, golden):
    import kernel as K
    q = torch.from_numpy(golden["fp4deq_q"]).to(dev)
    s = torch.from_numpy(golden["fp4deq_s"]).to(dev)
    out = K.dequant_fp4_weight(q, s).cpu().numpy()
    assert np.array_equal(bits(out), bits(golden["fp4deq_out"]))


def test_fp8_dequant_golden(dev, golden):
    import kernel as K
    b = torch.from_numpy(golden["fp8deq_b"]).to(dev)
    s = torch.from_numpy(golden["fp8deq_s"]).to(dev)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float32)
    try:
        out = K.weight_dequant(b, s).cpu().numpy()
    finally:
        torch.set_default_dtype(prev)
    assert np.array_equal(bits(out), bits(golden["fp8deq_out"]))


def test_fp4_dequant_all_codes_and_scales(dev):
    import kernel as K
    rng = np.random.default_rng(3)
    q = rng.integers(0, 256, (256, 128), dtype=np.uint8)
    s = rng.integers(0, 255, (256, 8), dtype=np.uint8)      # every finite e8m0 incl. 0 (2^-127)
    s[0, :] = np.arange(8)
    out = K.dequant_fp4_weight(torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev)).cpu().numpy()
    ref = F.dequant_fp4(q, s)
    assert np.array_equal(bits(out), bits(ref))


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("world", [1, 2, 4])
def test_store_pack_unpack_bit_exact(dev, fmt, world):
    """The packed resident store is lossless: unpack == reference dequant of the rank's slice."""
    from dsmoe import ExpertStore, synth
    H, I = 512, 512
    gen = torch.Generator().manual_seed(11)
    ew = synth.make_expert(fmt, H, I, gen)
    deq = F.dequant_fp8_block if fmt == "fp8" else F.dequant_fp4
    full = {n: deq(getattr(ew, n).numpy(), getattr(ew, "s" + n[1:]).numpy()) for n in ("w1", "w3", "w2")}
    for r in range(world):
        st = ExpertStore(fmt, H, I, 2, r, world, dev)
        st.pack(1, ew)
        w1, w3, w2 = (t.cpu().numpy() for t in st.unpack(1))
        sl = slice(r * I // world, (r + 1) * I // world)
        assert np.array_equal(bits(w1), bits(full["w1"][sl]))
        assert np.array_equal(bits(w3), bits(full["w3"][sl]))
        assert np.array_equal(bits(w2), bits(full["w2"][:, sl]))


# ------------------------------------------------------------------ router (indices bit-exact)

@pytest.mark.parametrize("sf,rs", [("sigmoid", 2.5), ("sqrtsoftplus", 1.5)])
def test_router_golden(dev, golden, sf, rs):
    from dsmoe import MoE, RouterWeights
    x, wg, bias = golden["rt_x"], golden["rt_wg"], golden["rt_bias"]
    m = MoE(x.shape[1], 64, wg.shape[0], 6, "fp8", sf, rs, device=dev)
    m.load_router(RouterWeights(torch.from_numpy(wg), torch.from_numpy(bias)))
    idx, wt, sc = m.route(torch.from_numpy(x).to(torch.bfloat16).to(dev))
    assert np.array_equal(idx.cpu().numpy(), golden[f"rt_{sf}_idx"])
    assert np.allclose(wt.cpu().numpy(), golden[f"rt_{sf}_wt"], rtol=1e-5)
    assert np.allclose(sc.cpu().numpy(), golden[f"rt_{sf}_sc"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("B", [1, 4, 8, 13, 64])
@pytest.mark.parametrize("sf", ["sigmoid", "sqrtsoftplus"])
def test_router_full_size(dev, B, sf):
    """384 experts x 5120 hidden, the benchmark's router: indices bit-exact vs the oracle."""
    from dsmoe import MoE, make_router, make_tokens
    gen = torch.Generator().manual_seed(100 + B)
    rw = make_router(384, 5120, gen)
    x = make_tokens(B, 5120, gen)
    m = MoE(5120, 64, 384, 6, "fp8", sf, 2.5, device=dev)
    m.load_router(rw)
    idx, wt, sc = m.route(x.to(dev))
    ridx, rwt, rsc = OM.route(x.float().numpy(), rw.wg.numpy(), rw.bias.numpy(), 6, sf, 2.5)
    # A token whose 6th and 7th biased scores lie within 1e-6 could flip between two correct
    # orderings; on these seeds no token comes that close, so every index is compared bit-exact.
    tie = OM.near_tie(x.float().numpy(), rw.wg.numpy(), rw.bias.numpy(), 6, sf, eps=1e-6)
    assert int(tie.sum()) == 0, f"{int(tie.sum())} near-tie tokens: pick other seeds"
    ok = (idx.cpu().numpy() == ridx).all(axis=1)
    assert ok.all(), f"index mismatch on tokens {np.nonzero(~ok)[0]}"
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), rsc.view(np.uint32)) or \
        np.allclose(sc.cpu().numpy(), rsc, rtol=2e-7, atol=0)
    assert np.allclose(wt.cpu().numpy(), rwt, rtol=1e-6)


def test_router_image_mask_bias_vl(dev):
    from dsmoe import MoE, RouterWeights
    gen = torch.Generator().manual_seed(9)
    H, E, B = 512, 64, 6
    wg = torch.randn((E, H), generator=gen) * 0.02
    bias = torch.randn((E,), generator=gen) * 0.01
    bias_vl = torch.randn((E,), generator=gen) * 0.5
    x = torch.randn((B, H), generator=gen).to(torch.bfloat16)
    mask = torch.tensor([0, 1, 0, 1, 1, 0], dtype=torch.bool)
    m = MoE(H, 64, E, 6, "fp8", "sigmoid", 2.5, device=dev)
    m.load_router(RouterWeights(wg, bias, bias_vl))
    idx, wt, _ = m.route(x.to(dev), mask.to(dev))
    ridx, rwt, _ = OM.route(x.float().numpy(), wg.numpy(), bias.numpy(), 6, "sigmoid", 2.5,
                            bias_vl.numpy(), mask.numpy())
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.allclose(wt.cpu().numpy(), rwt, rtol=1e-6)


# ------------------------------------------------------------------ layer outputs (tolerance)

def test_moe_layer_golden(dev, golden):
    """The small layers computed by the reference's own shim linears (tests/golden)."""
    from dsmoe import MoE, RouterWeights
    from dsmoe.synth import ExpertWeights
    for fmt in ("fp8", "fp4"):
        pre = f"moe_{fmt}_"
        wg, bias, x = golden[pre + "wg"], golden[pre + "bias"], golden[pre + "x"]
        E, H = wg.shape
        I = golden[f"{pre}e0_w1"].shape[0]
        m = MoE(H, I, E, 6, fmt, "sigmoid", 2.5, device=dev)
        m.load_router(RouterWeights(torch.from_numpy(wg), torch.from_numpy(bias)))

        def ew(j, f):
            g = lambda n: torch.from_numpy(np.ascontiguousarray(golden[f"{pre}e{j}_{n}"]))
            return ExpertWeights(f, g("w1"), g("s1"), g("w3"), g("s3"), g("w2"), g("s2"))

        for j in range(E):
            m.load_expert(j, ew(j, fmt))
        m.load_shared(ew(E, "fp8"))
        xt = torch.from_numpy(x).to(torch.bfloat16).to(dev)
        idx, wt, _ = m.route(xt)
        assert np.array_equal(idx.cpu().numpy(), golden[pre + "idx"])
        y = bf16_np(m.forward(xt))
        mar, cos = OM.compare(y, golden[pre + "y"])
        assert mar < MAR_TOL and cos > COS_TOL, (fmt, mar, cos)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("B", [1, 3, 8, 13, 64])
def test_moe_layer_vs_oracle(dev, fmt, B):
    spec = make_layer_cpu(fmt, 1024, 512, 32, seed=1000 + B)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    gen = torch.Generator().manual_seed(B)
    x = torch.randn((B, 1024), generator=gen).to(torch.bfloat16)
    idx = torch.empty((B, 6), dtype=torch.int64, device=dev)
    wt = torch.empty((B, 6), dtype=torch.float32, device=dev)
    part = m.partial(x.to(dev), idx=idx, wt=wt)
    y = bf16_np(m.forward(x.to(dev)))
    yr, ridx, rwt = OM.moe_forward(ref, x.float().numpy())
    assert np.array_equal(idx.cpu().numpy(), ridx)
    mar, cos = OM.compare(y, yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
    # fp32 partial (no bf16 rounding) is much closer
    yp, _, _ = OM.moe_forward(ref, x.float().numpy(), return_partial=True)
    mar32, cos32 = OM.compare(part.cpu().numpy(), yp)
    assert mar32 < 2e-3 and cos32 > 0.99999, (mar32, cos32)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_moe_skewed_routing_virtual_slots(dev, fmt):
    """Every token picks the same few experts: an expert's 64 tokens span 8 slots of 8."""
    spec = make_layer_cpu(fmt, 512, 256, 16, seed=77)
    spec["router"].bias[:6] += 10.0           # experts 0..5 win for every token
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    x = torch.randn((64, 512), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    y = bf16_np(m.forward(x.to(dev)))
    yr, ridx, _ = OM.moe_forward(ref, x.float().numpy())
    assert (np.sort(ridx, axis=1) == np.arange(6)).all()
    mar, cos = OM.compare(y, yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("world", [2, 8])
def test_tp_partials_on_one_gpu(dev, fmt, world):
    """Tensor-parallel slices (I/world rows per rank) built side by side: partials sum to the layer."""
    spec = make_layer_cpu(fmt, 512, 512, 16, seed=21)
    ref = to_oracle_layer(spec)
    x = torch.randn((4, 512), generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    tot = None
    for r in range(world):
        m = to_gpu_moe(spec, rank=r, world=world, device=dev)
        p = m.partial(x.to(dev)).cpu().numpy().astype(np.float64)
        pr, _, _ = OM.moe_forward(ref, x.float().numpy(), r, world, return_partial=True)
        mar, cos = OM.compare(p, pr)
        assert mar < 2e-3 and cos > 0.99999, (r, mar, cos)
        tot = p if tot is None else tot + p
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    mar, cos = OM.compare(F.bf16_round(tot.astype(np.float32)), yr)
    assert mar < MAR_TOL and cos > COS_TOL


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_full_size_layer(dev, fmt):
    """The benchmark layer at full size (H 5120, I 2048, 384 experts + shared), generated on the GPU,
    at decode batches 1, 4 and 8 (configs C1 / C2): the routed experts those tokens choose and the
    shared expert are kept on the CPU and checked against the oracle."""
    from dsmoe import MoE, make_expert, make_router, make_tokens
    gen = torch.Generator(device=dev).manual_seed(2024)
    H, I, E = 5120, 2048, 384
    m = MoE(H, I, E, 6, fmt, "sigmoid", 2.5, device=dev, max_tokens=8)
    rw = make_router(E, H, gen, device=dev)
    m.load_router(rw)
    shared = make_expert("fp8", H, I, gen, device=dev)
    m.load_shared(shared)
    kept = {}
    batches = ((0, 1), (1, 5), (5, 13))  # B = 1, 4, 8
    x = make_tokens(13, H, gen, device=dev)
    ridx_all, _, _ = OM.route(x.float().cpu().numpy(), rw.wg.cpu().numpy(), rw.bias.cpu().numpy())
    need = set(ridx_all.ravel().tolist())
    for e in range(E):
        ew = make_expert(fmt, H, I, gen, device=dev)
        m.load_expert(e, ew)
        if e in need:
            kept[e] = ew.to("cpu")
        del ew
    from _util import to_oracle_expert
    experts = [to_oracle_expert(kept[e]) if e in kept else None for e in range(E)]
    ref = OM.MoELayer(rw.wg.cpu().numpy(), rw.bias.cpu().numpy(), experts, to_oracle_expert(shared.to("cpu")))
    for b0, b1 in batches:
        xb = x[b0:b1]
        y = bf16_np(m.forward(xb))
        yr, ridx, _ = OM.moe_forward(ref, xb.float().cpu().numpy())
        idx, _, _ = m.route(xb)
        assert np.array_equal(idx.cpu().numpy(), ridx)
        mar, cos = OM.compare(y, yr)
        assert mar < MAR_TOL and cos > COS_TOL, (b1 - b0, mar, cos)
    m.check(8)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("B", [1, 5])
def test_outlier_channels(dev, fmt, B):
    """Hidden states with a few outlier channels (4 channels at 300x the rest, as real residual
    streams have) go through the per-token power-of-two pre-scale and the e4m3 hi / lo split, and
    drive many gate / up values into the SwiGLU clamps, so h mixes clamped and small values: the
    layer must stay within the north-star tolerance of the oracle."""
    spec = make_layer_cpu(fmt, 1024, 512, 32, seed=3100 + B)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    x = torch.randn((B, 1024), generator=torch.Generator().manual_seed(31 + B))
    x[:, [7, 300, 555, 1000]] *= 300.0
    x = x.to(torch.bfloat16)
    y = bf16_np(m.forward(x.to(dev)))
    yr, ridx, _ = OM.moe_forward(ref, x.float().numpy())
    idx, _, _ = m.route(x.to(dev))
    assert np.array_equal(idx.cpu().numpy(), ridx)
    mar, cos = OM.compare(y, yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
    m.check(B)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_real_width_tp8_slices(dev, fmt):
    """The real model's intermediate width, 2304, split over 8 ranks: 288 rows per rank, so FP8
    128-row scale blocks straddle the slices (dsv41/ref/fp4lib.c:114-115, dsv41/tt/moe.py:42-45).
    Every rank's partial matches the oracle's partial of the same rows; the partials sum to the layer."""
    spec = make_layer_cpu(fmt, 1024, 2304, 16, seed=2304)
    ref = to_oracle_layer(spec)
    x = torch.randn((3, 1024), generator=torch.Generator().manual_seed(288)).to(torch.bfloat16)
    tot = None
    for r in range(8):
        m = to_gpu_moe(spec, rank=r, world=8, device=dev)
        assert m.routed.inter_local == 288
        p = m.partial(x.to(dev)).cpu().numpy().astype(np.float64)
        m.check(3)
        pr, _, _ = OM.moe_forward(ref, x.float().numpy(), r, 8, return_partial=True)
        mar, cos = OM.compare(p, pr)
        assert mar < 2e-3 and cos > 0.99999, (r, mar, cos)
        tot = p if tot is None else tot + p
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    mar, cos = OM.compare(F.bf16_round(tot.astype(np.float32)), yr)
    assert mar < MAR_TOL and cos > COS_TOL


# ------------------------------------------------------------------ kernel.py surface

def test_kernel_surface_gemms_golden(dev, golden):
    import kernel as K
    x = torch.from_numpy(golden["gemm_x"]).to(torch.bfloat16).to(dev)
    a, a_s = x.float(), torch.ones((x.shape[0], x.shape[1] // 128), device=dev)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        y8 = K.fp8_gemm(a, a_s, torch.from_numpy(golden["gemm_q8"]).to(dev).view(torch.float8_e4m3fn),
                        torch.from_numpy(golden["gemm_s8"]).to(dev))
        y4 = K.fp4_gemm(a, a_s, torch.from_numpy(golden["gemm_q4"]).to(dev),
                        torch.from_numpy(golden["gemm_s4"]).to(dev))
    finally:
        torch.set_default_dtype(prev)
    assert y8.dtype == torch.bfloat16 and y4.dtype == torch.bfloat16
    for y, key in ((y8, "gemm_y8"), (y4, "gemm_y4")):
        ref = golden[key]
        d = np.abs(y.float().cpu().numpy() - ref)
        assert np.all(d <= np.abs(ref) * 2.0 ** -7 + 1e-6), float(d.max())


def test_kernel_surface_fakequant_gemm(dev):
    """e4m3 activations with per-128 scales (the shim's fake-quant mode) through fp8_gemm."""
    import kernel as K
    gen = torch.Generator().manual_seed(4)
    x = (torch.randn((5, 384), generator=gen) * 2).to(torch.bfloat16)
    from dsmoe.synth import quant_fp8_block
    q, s = quant_fp8_block(torch.randn((200, 384), generator=gen) * 0.02)
    xs = x.float().view(5, 3, 128)
    amax = xs.abs().amax(-1, keepdim=True).clamp(min=1e-4)
    sa = amax / 448.0
    qa = (xs / sa).clamp(-448, 448).to(torch.float8_e4m3fn).view(5, 384)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float32)
    try:
        y = K.fp8_gemm(qa.to(dev), sa.squeeze(-1).to(dev), q.to(dev).view(torch.float8_e4m3fn), s.to(dev))
    finally:
        torch.set_default_dtype(prev)
    ref = (qa.float().view(5, 3, 128) * sa).view(5, 384).double() @ torch.from_numpy(
        F.dequant_fp8_block(q.numpy(), s.numpy())).double().T
    assert torch.allclose(y.cpu().double(), ref, rtol=1e-4, atol=1e-5)


def test_act_quant_golden(dev, golden):
    x = torch.from_numpy(golden["actq_x"]).to(torch.bfloat16).to(dev)
    from dsmoe import _lib as L
    for key, pow2 in (("actq_on", 0), ("actq_pow2", 1)):
        q = torch.empty(x.shape, dtype=torch.uint8, device=dev)
        s = torch.empty((x.shape[0], x.shape[1] // 128), dtype=torch.float32, device=dev)
        L.call("dsmoe_act_quant", L.ptr(x), L.DTYPE_BF16, x.shape[0], x.shape[1], 128, pow2, L.ptr(q), L.ptr(s),
               L.stream_of(x))
        assert np.array_equal(q.cpu().numpy(), golden[key])
        assert np.array_equal(s.cpu().numpy(), golden[key + "_s"])


def test_expert_class_vs_oracle(dev):
    from dsmoe import Expert, synth
    gen = torch.Generator().manual_seed(8)
    for fmt in ("fp8", "fp4"):
        ew = synth.make_expert(fmt, 512, 256, gen)
        x = torch.randn((3, 512), generator=gen).to(torch.bfloat16)
        w = torch.rand((3,), generator=gen)
        y = Expert(ew, dev)(x.to(dev), w.to(dev)).cpu().numpy()
        from _util import to_oracle_expert
        yr = OM.expert_ffn(x.float().numpy(), to_oracle_expert(ew), w.numpy())
        mar, cos = OM.compare(y, yr)
        assert mar < 1e-3 and cos > 0.99999, (fmt, mar, cos)


# ------------------------------------------------------------------ boundary behaviour

def test_errors_are_raised_not_launched(dev):
    from dsmoe import MoE, _lib as L
    m = MoE(512, 256, 16, 6, "fp8", device=dev)
    with pytest.raises(ValueError):
        m.forward(torch.zeros((2, 256), dtype=torch.bfloat16, device=dev))      # wrong hidden
    with pytest.raises(TypeError):
        m.forward(torch.zeros((2, 512), dtype=torch.float32, device=dev))       # wrong dtype
    with pytest.raises(L.DsmoeError) as ei:
        L.call("dsmoe_moe_decode", m._layer, L.ptr(torch.zeros((1, 512), dtype=torch.bfloat16, device=dev)),
               1, None, L.ptr(torch.zeros((1, 512), device=dev)), L.DTYPE_F32, None, None, None,
               L.ptr(m.workspace), 16, L.stream_of())                            # workspace too small
    assert ei.value.code == L.ERR_WORKSPACE
    with pytest.raises(L.DsmoeError) as ei:
        L.call("dsmoe_moe_decode", m._layer, L.ptr(torch.zeros((1, 512), dtype=torch.bfloat16, device=dev)),
               65, None, None, L.DTYPE_F32, None, None, None, L.ptr(m.workspace), m.workspace.numel(),
               L.stream_of())                                                    # batch too large
    assert ei.value.code == L.ERR_ARG
    torch.cuda.synchronize()


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_workspace_reuse_across_calls_and_batches(dev, fmt):
    """One workspace, many calls: the persistent path (B <= 8) and the multi-kernel path (B > 8)
    alternate; every output matches the oracle and no bounded wait expires."""
    spec = make_layer_cpu(fmt, 1024, 256, 32, seed=55)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    gen = torch.Generator().manual_seed(12)
    for B in (1, 8, 13, 2, 1, 64, 5, 1, 1):
        x = torch.randn((B, 1024), generator=gen).to(torch.bfloat16)
        y = bf16_np(m.forward(x.to(dev)))
        yr, _, _ = OM.moe_forward(ref, x.float().numpy())
        mar, cos = OM.compare(y, yr)
        assert mar < MAR_TOL and cos > COS_TOL, (B, mar, cos)
    m.check(8)
