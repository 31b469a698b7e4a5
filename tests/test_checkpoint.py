"""Checkpoint loader (dsmoe.checkpoint) on a synthetic two-shard safetensors checkpoint in the
DeepSeek-V4.1-Flash layout (dsv41/ckpt.py:3-6, 41-50; dsv41/tt/weights.py:45-61, 136-143):
routed experts packed e2m1 + e8m0, shared expert e4m3 + e8m0 128 x 128 block scales, fp32 router.
CPU: the reader returns the stored bytes, shapes and exact scales. GPU: a layer filled from the
checkpoint computes exactly what the same weights loaded directly compute, and matches the oracle."""
import json
import os

import numpy as np
import pytest
import torch

from _util import bf16_np

H, I, E, LAYER = 512, 256, 4, 3


def _shared_fp8_e8m0(w: torch.Tensor):
    """e4m3 with a power-of-two scale per 128 x 128 block (the checkpoint's non-expert format)."""
    o, i = w.shape
    q = torch.empty((o, i), dtype=torch.uint8)
    sb = torch.empty((-(-o // 128), -(-i // 128)), dtype=torch.uint8)
    for a in range(0, o, 128):
        for b in range(0, i, 128):
            blk = w[a:a + 128, b:b + 128]
            e = int(torch.ceil(torch.log2(blk.abs().max().clamp_min(1e-30) / 448.0)).item())
            sb[a // 128, b // 128] = e + 127
            q[a:a + 128, b:b + 128] = (blk / 2.0 ** e).to(torch.float8_e4m3fn).view(torch.uint8)
    return q, sb


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from dsmoe import synth
    from dsmoe.checkpoint import write_safetensors
    d = tmp_path_factory.mktemp("ckpt")
    gen = torch.Generator().manual_seed(99)
    f = f"layers.{LAYER}.ffn"
    shards = [{}, {}]
    truth = {"experts": []}
    for e in range(E):
        parts = {}
        for pj, shape in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I))):
            q, s = synth.quant_fp4_e8m0(torch.randn(shape, generator=gen) * 0.02)
            shards[e % 2][f"{f}.experts.{e}.{pj}.weight"] = (q.numpy(), "I8")
            shards[e % 2][f"{f}.experts.{e}.{pj}.scale"] = (s.numpy(), "F8_E8M0")
            parts[pj] = (q, s)
        truth["experts"].append(parts)
    sh = {}
    for pj, shape in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I))):
        q, sb = _shared_fp8_e8m0(torch.randn(shape, generator=gen) * 0.02)
        shards[0][f"{f}.shared_experts.{pj}.weight"] = (q.numpy(), "F8_E4M3")
        shards[0][f"{f}.shared_experts.{pj}.scale"] = (sb.numpy(), "F8_E8M0")
        sh[pj] = (q, sb)
    truth["shared"] = sh
    wg = torch.randn((E, H), generator=gen) * 0.02
    bias = torch.randn((E,), generator=gen) * 0.01
    shards[1][f"{f}.gate.weight"] = (wg.numpy(), "F32")
    shards[1][f"{f}.gate.bias"] = (bias.numpy(), "F32")
    truth["router"] = (wg, bias)
    wm = {}
    for k, t in enumerate(shards):
        fn = f"model-0000{k + 1}-of-00002.safetensors"
        write_safetensors(os.path.join(d, fn), t)
        wm.update({name: fn for name in t})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as fh:
        json.dump({"metadata": {}, "weight_map": wm}, fh)
    return str(d), truth


def test_reader_returns_checkpoint_bytes(ckpt):
    from dsmoe.checkpoint import SafetensorsCheckpoint, router, routed_expert, shared_expert
    path, truth = ckpt
    ck = SafetensorsCheckpoint(path)
    for e in range(E):
        ew = routed_expert(ck, LAYER, e)
        assert ew.fmt == "fp4"
        for pj, (q, s) in truth["experts"][e].items():
            assert torch.equal(getattr(ew, pj), q) and torch.equal(getattr(ew, "s" + pj[1]), s)
    sh = shared_expert(ck, LAYER)
    assert sh.fmt == "fp8"
    for pj, (q, sb) in truth["shared"].items():
        assert torch.equal(getattr(sh, pj), q)
        exact = torch.ldexp(torch.ones(sb.shape), sb.to(torch.int32) - 127)
        assert torch.equal(getattr(sh, "s" + pj[1]), exact)
    rw = router(ck, LAYER)
    assert torch.equal(rw.wg, truth["router"][0]) and torch.equal(rw.bias, truth["router"][1])
    assert rw.bias_vl is None
    ck.close()


def test_reader_rejects_wrong_formats(tmp_path):
    from dsmoe.checkpoint import SafetensorsCheckpoint, routed_expert, write_safetensors
    p = tmp_path / "one.safetensors"
    write_safetensors(str(p), {"layers.0.ffn.experts.0.w1.weight": (np.zeros((8, 16), np.uint8), "F8_E4M3"),
                               "layers.0.ffn.experts.0.w1.scale": (np.zeros((8, 1), np.uint8), "F8_E8M0")})
    with pytest.raises(ValueError, match="packed e2m1"):
        routed_expert(SafetensorsCheckpoint(str(p)), 0, 0)


@pytest.mark.gpu
def test_layer_from_checkpoint_matches_direct_load(ckpt):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dsmoe import MoE
    from dsmoe.checkpoint import SafetensorsCheckpoint, load_layer, router, routed_expert, shared_expert
    from oracle import moe as OM
    from _util import to_oracle_layer
    path, _ = ckpt
    dev = torch.device("cuda", 0)
    ck = SafetensorsCheckpoint(path)
    a = MoE(H, I, E, 2, "fp4", "sigmoid", 2.5, device=dev)
    load_layer(a, ck, LAYER)
    b = MoE(H, I, E, 2, "fp4", "sigmoid", 2.5, device=dev)
    b.load_router(router(ck, LAYER))
    b.load_shared(shared_expert(ck, LAYER))
    experts = [routed_expert(ck, LAYER, e) for e in range(E)]
    for e, ew in enumerate(experts):
        b.load_expert(e, ew)
    x = torch.randn((3, H), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(dev)
    ya, yb = a.forward(x), b.forward(x)
    assert torch.equal(ya, yb)
    spec = dict(fmt="fp4", hidden=H, inter=I, n_experts=E, topk=2, score_func="sigmoid", route_scale=2.5,
                experts=experts, shared=shared_expert(ck, LAYER), router=router(ck, LAYER))
    yr, _, _ = OM.moe_forward(to_oracle_layer(spec), x.float().cpu().numpy())
    mar, cos = OM.compare(bf16_np(ya), yr)
    assert mar < 1e-2 and cos > 0.9999, (mar, cos)
    ck.close()
