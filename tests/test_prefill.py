"""Prefill / batched layer on the tcgen05 grouped GEMMs (dsmoe_moe_prefill) against the oracle.

Routing is either the layer's router (indices must match the oracle bit for bit, as in decode) or
forced (a Zipf-skewed draw, the prefill benchmark's routing), in which case the oracle takes the
same idx / wt (oracle.moe.moe_forward_routed restates dsv41/tt/moe.py:182-200, 263-288).
Tolerances: bf16 output max-abs-rel <= 1e-2 and cosine >= 0.9999; the fp32
partial (no bf16 rounding) within 2e-3."""
import numpy as np
import pytest
import torch

from _util import bf16_np, make_layer_cpu, to_gpu_moe, to_oracle_layer

pytestmark = pytest.mark.gpu

MAR_TOL, COS_TOL = 1e-2, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401  (fails loudly if libdsmoe.so is missing)
    return torch.device("cuda", 0)


def _om():
    from oracle import moe as OM
    return OM


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("P", [1, 13, 77])
def test_prefill_router_vs_oracle(dev, fmt, P):
    OM = _om()
    spec = make_layer_cpu(fmt, 1024, 512, 32, seed=5000 + P)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    x = torch.randn((P, 1024), generator=torch.Generator().manual_seed(P)).to(torch.bfloat16)
    y = m.prefill(x.to(dev))
    m.prefill_check(P)
    yr, ridx, _ = OM.moe_forward(ref, x.float().numpy())
    idx, _, _ = m.route(x.to(dev))
    assert np.array_equal(idx.cpu().numpy(), ridx)
    mar, cos = OM.compare(bf16_np(y), yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
    part = m.prefill(x.to(dev), partial=True)
    yp, _, _ = OM.moe_forward(ref, x.float().numpy(), return_partial=True)
    mar32, cos32 = OM.compare(part.cpu().numpy(), yp)
    assert mar32 < 2e-3 and cos32 > 0.99999, (mar32, cos32)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_prefill_zipf_forced_routing(dev, fmt):
    """126 tokens, Zipf(1.1) over 64 experts: popular experts span several 64-token chunks."""
    from dsmoe import zipf_routing
    OM = _om()
    spec = make_layer_cpu(fmt, 1024, 256, 64, seed=77)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    gen = torch.Generator().manual_seed(126)
    x = torch.randn((126, 1024), generator=gen).to(torch.bfloat16)
    idx, wt = zipf_routing(126, 64, 6, gen)
    counts = np.bincount(idx.numpy().ravel(), minlength=64)
    assert counts.max() > 64  # at least one expert needs two chunks
    y = m.prefill(x.to(dev), idx, wt)
    m.prefill_check(126)
    yr = OM.moe_forward_routed(ref, x.float().numpy(), idx.numpy(), wt.numpy())
    mar, cos = OM.compare(bf16_np(y), yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_prefill_tp_partials(dev, fmt):
    """Tensor-parallel slices (I / 2 rows per rank) built side by side: prefill partials sum to the layer."""
    OM = _om()
    spec = make_layer_cpu(fmt, 512, 512, 16, seed=23)
    ref = to_oracle_layer(spec)
    x = torch.randn((20, 512), generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    tot = None
    for r in range(2):
        m = to_gpu_moe(spec, rank=r, world=2, device=dev)
        p = m.prefill(x.to(dev), partial=True).cpu().numpy().astype(np.float64)
        pr, _, _ = OM.moe_forward(ref, x.float().numpy(), r, 2, return_partial=True)
        mar, cos = OM.compare(p, pr)
        assert mar < 2e-3 and cos > 0.99999, (r, mar, cos)
        tot = p if tot is None else tot + p
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    from oracle.formats import bf16_round
    mar, cos = OM.compare(bf16_round(tot.astype(np.float32)), yr)
    assert mar < MAR_TOL and cos > COS_TOL


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_prefill_full_width(dev, fmt):
    """The benchmark's expert shapes (H 5120, I 2048) with 16 experts and 64 tokens."""
    OM = _om()
    spec = make_layer_cpu(fmt, 5120, 2048, 16, seed=31)
    m = to_gpu_moe(spec, device=dev)
    ref = to_oracle_layer(spec)
    x = torch.randn((64, 5120), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    y = m.prefill(x.to(dev))
    m.prefill_check(64)
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    mar, cos = OM.compare(bf16_np(y), yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)


def test_prefill_matches_decode(dev):
    """The same tokens through the decode path (B <= 64) and the prefill path agree closely."""
    OM = _om()
    spec = make_layer_cpu("fp8", 1024, 512, 32, seed=41)
    m = to_gpu_moe(spec, device=dev)
    x = torch.randn((48, 1024), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(dev)
    a = m.partial(x).cpu().numpy()
    b = m.prefill(x, partial=True).cpu().numpy()
    mar, cos = OM.compare(b, a)
    assert mar < 2e-3 and cos > 0.99999, (mar, cos)


def test_prefill_bad_index_is_reported(dev):
    from dsmoe._lib import DsmoeError
    spec = make_layer_cpu("fp8", 512, 256, 16, seed=5)
    m = to_gpu_moe(spec, device=dev)
    x = torch.randn((4, 512), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(dev)
    idx = torch.tensor([[0, 1, 2, 3, 4, 99]] * 4, dtype=torch.int64)
    wt = torch.full((4, 6), 0.4)
    m.prefill(x, idx, wt)
    with pytest.raises(DsmoeError, match="out of range"):
        m.prefill_check(4)
    m.prefill(x, idx.clamp(max=15), wt)  # the next call is clean
    m.prefill_check(4)
