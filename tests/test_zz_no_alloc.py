"""dsmoe_router_noalloc (scratch in the library's own device array) against dsmoe_router (caller
workspace), through the C ABI. Collected last on purpose: it must pass after every other test has
used the device, as well as on its own."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401  (fails loudly if libdsmoe.so is missing)
    return torch.device("cuda", 0)


def _noalloc(m, x, image_mask=None):
    from dsmoe import _lib as L
    B = x.shape[0]
    idx = torch.empty((B, m.topk), dtype=torch.int64, device=x.device)
    wt = torch.empty((B, m.topk), dtype=torch.float32, device=x.device)
    sc = torch.empty((B, m.n_experts), dtype=torch.float32, device=x.device)
    L.call("dsmoe_router_noalloc", m._layer, L.ptr(x), B, L.ptr(image_mask), L.ptr(idx), L.ptr(wt), L.ptr(sc),
           L.stream_of(x))
    return idx, wt, sc


@pytest.mark.parametrize("B,sf", [(1, "sigmoid"), (5, "sqrtsoftplus"), (64, "sigmoid")])
def test_noalloc_router_matches_workspace_router(dev, B, sf):
    from dsmoe import MoE, make_router, make_tokens
    gen = torch.Generator().manual_seed(7000 + B)
    m = MoE(5120, 64, 384, 6, "fp8", sf, 2.5, device=dev)
    m.load_router(make_router(384, 5120, gen))
    x = make_tokens(B, 5120, gen).to(dev)
    idx0, wt0, sc0 = m.route(x)
    for _ in range(2):  # two calls in a row on the same static scratch
        idx1, wt1, sc1 = _noalloc(m, x)
        torch.cuda.synchronize()
        assert torch.equal(idx1, idx0)
        assert torch.allclose(wt1, wt0, rtol=1e-6, atol=0)
        assert torch.allclose(sc1, sc0, rtol=1e-6, atol=0)


def test_noalloc_router_image_mask(dev):
    from dsmoe import MoE, RouterWeights
    gen = torch.Generator().manual_seed(71)
    H, E, B = 512, 64, 6
    rw = RouterWeights(torch.randn((E, H), generator=gen) * 0.02, torch.randn((E,), generator=gen) * 0.01,
                       torch.randn((E,), generator=gen) * 0.5)
    m = MoE(H, 64, E, 6, "fp8", "sigmoid", 2.5, device=dev)
    m.load_router(rw)
    x = torch.randn((B, H), generator=gen).to(torch.bfloat16).to(dev)
    mask = torch.tensor([0, 1, 0, 1, 1, 0], dtype=torch.uint8, device=dev)
    idx0, wt0, _ = m.route(x, mask)
    idx1, wt1, _ = _noalloc(m, x, mask)
    assert torch.equal(idx1, idx0)
    assert torch.allclose(wt1, wt0, rtol=1e-6, atol=0)


def test_noalloc_router_rejects_beyond_limits(dev):
    from dsmoe import MoE, make_router, make_tokens
    from dsmoe._lib import DsmoeError
    gen = torch.Generator().manual_seed(72)
    m = MoE(5120, 64, 384, 6, "fp8", "sigmoid", 2.5, device=dev, max_tokens=64)
    m.load_router(make_router(384, 5120, gen))
    x = make_tokens(65, 5120, gen).to(dev)
    with pytest.raises(DsmoeError, match="scratch limit"):
        _noalloc(m, x)
    big = MoE(8192 + 128, 64, 16, 6, "fp8", "sigmoid", 2.5, device=dev)
    big.load_router(make_router(16, 8192 + 128, gen))
    with pytest.raises(DsmoeError, match="scratch limit"):
        _noalloc(big, make_tokens(1, 8192 + 128, gen).to(dev))
