"""The DSpark draft model's MoE (dsv41/tt/dspark.py:61-104): 128 routed experts, top-3 of
sqrt(softplus) scores plus bias, weights normalised and scaled by ROUTE_SCALE 1.5 (dsv41/tt/moe.py:15),
FP4 experts plus the shared expert, on a verify block of 5 tokens (BLOCK, dspark.py:23). The same
layer kernels serve it: the persistent decode kernel for the block, the tcgen05 prefill path for a
longer draft, both against the oracle."""
import numpy as np
import pytest
import torch

from _util import bf16_np, make_layer_cpu, to_gpu_moe, to_oracle_layer

pytestmark = pytest.mark.gpu

MAR_TOL, COS_TOL = 1e-2, 0.9999
NEXP_D, TOPK_D, ROUTE_SCALE_D, BLOCK = 128, 3, 1.5, 5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401  (fails loudly if libdsmoe.so is missing)
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def layer(dev):
    spec = make_layer_cpu("fp4", 1024, 512, NEXP_D, seed=128, topk=TOPK_D, score_func="sqrtsoftplus",
                          route_scale=ROUTE_SCALE_D)
    return spec, to_gpu_moe(spec, device=dev), to_oracle_layer(spec)


def test_dspark_verify_block(dev, layer):
    from oracle import moe as OM
    spec, m, ref = layer
    x = torch.randn((BLOCK, 1024), generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    idx, wt, _ = m.route(x.to(dev))
    y = m.forward(x.to(dev))
    m.check(BLOCK)
    yr, ridx, rwt = OM.moe_forward(ref, x.float().numpy())
    assert idx.shape == (BLOCK, TOPK_D)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.allclose(wt.cpu().numpy(), rwt, rtol=1e-6, atol=0)
    assert np.allclose(wt.sum(1).cpu().numpy(), ROUTE_SCALE_D, rtol=1e-5)
    mar, cos = OM.compare(bf16_np(y), yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)


def test_dspark_longer_draft_prefill(dev, layer):
    from oracle import moe as OM
    spec, m, ref = layer
    x = torch.randn((40, 1024), generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    y = m.prefill(x.to(dev))
    m.prefill_check(40)
    yr, _, _ = OM.moe_forward(ref, x.float().numpy())
    mar, cos = OM.compare(bf16_np(y), yr)
    assert mar < MAR_TOL and cos > COS_TOL, (mar, cos)
