"""The traced decode step (dsmoe.DecodeTrace, the role of the reference's DecodeTrace in
dsv41/tt/model.py:262-330): the decode calls of a set of layers replayed as one CUDA graph, with the
tokens copied in from pinned host memory and the outputs copied out inside the graph.

Every replay must give the bits MoE.forward gives on the same tokens (both stores' kernels are
deterministic), match the oracle within the layer tests' bars, follow new host tokens from step
to step, and leave the layers usable eagerly afterwards."""
import numpy as np
import pytest
import torch

from oracle import moe as OM

from _util import make_layer_cpu, to_gpu_moe, to_oracle_layer

pytestmark = pytest.mark.gpu

MAR_TOL, COS_TOL = 1e-2, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def layers(dev):
    specs = [make_layer_cpu(fmt, 1024, 512, 32, seed=7100 + i) for i, fmt in enumerate(("fp8", "fp4", "fp8"))]
    return specs, [to_gpu_moe(s, device=dev) for s in specs]


@pytest.mark.parametrize("B", [1, 5, 8])
@pytest.mark.parametrize("store", ["tc", "frag"])
def test_trace_matches_forward_and_oracle(dev, layers, B, store):
    from dsmoe import DecodeTrace
    specs, ms = layers
    for m in ms:
        m.use_decode_store(store)
    try:
        tr = DecodeTrace(ms, B)
        g = torch.Generator().manual_seed(B)
        for step in range(3):
            x = torch.randn((len(ms), B, 1024), generator=g).to(torch.bfloat16)
            y = tr.step(x).clone()
            tr.check()
            for i, (spec, m) in enumerate(zip(specs, ms)):
                y_e = m.forward(x[i].to(dev)).cpu()
                assert torch.equal(y[i], y_e), (store, B, step, i)
                if step == 2:
                    yr, _, _ = OM.moe_forward(to_oracle_layer(spec), x[i].float().numpy())
                    mar, cos = OM.compare(y[i].float().numpy(), yr)
                    assert mar < MAR_TOL and cos > COS_TOL, (store, B, i, mar, cos)
        tr.release()
        with pytest.raises(RuntimeError):
            tr.step()
    finally:
        for m in ms:
            m.use_decode_store("tc")


def test_trace_inputs_follow_host_buffer(dev, layers):
    """Writing x_host directly (no argument to step) is read by the next replay."""
    from dsmoe import DecodeTrace
    _, ms = layers
    tr = DecodeTrace(ms[:2], 2)
    g = torch.Generator().manual_seed(11)
    outs = []
    for _ in range(2):
        tr.x_host.copy_(torch.randn((2, 2, 1024), generator=g).to(torch.bfloat16))
        outs.append(tr.step().clone())
    assert not torch.equal(outs[0], outs[1])
    assert np.isfinite(outs[1].float().numpy()).all()
    tr.release()


def test_forward_out_argument(dev, layers):
    _, ms = layers
    x = torch.randn((3, 1024), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(dev)
    out = torch.empty((3, 1024), dtype=torch.bfloat16, device=dev)
    y = ms[0].forward(x, out=out)
    assert y.data_ptr() == out.data_ptr()
    assert torch.equal(out, ms[0].forward(x))
    with pytest.raises(ValueError):
        ms[0].forward(x, out=torch.empty((3, 1024), dtype=torch.float32, device=dev))
    with pytest.raises(ValueError):
        ms[0].forward(x, out=torch.empty((2, 1024), dtype=torch.bfloat16, device=dev))


def test_trace_rejects_bad_arguments(dev, layers):
    from dsmoe import DecodeTrace
    _, ms = layers
    with pytest.raises(ValueError):
        DecodeTrace([], 1)
    with pytest.raises(ValueError):
        DecodeTrace(ms, 0)
    with pytest.raises(ValueError):
        DecodeTrace(ms, ms[0].max_tokens + 1)
