"""Shared helpers for the parity tests: seeded layers built once on the CPU, handed to both the
CUDA path (dsmoe) and the oracle, so both see the same bytes."""
import numpy as np
import torch

from oracle import moe as OM


def make_layer_cpu(fmt, hidden, inter, n_experts, seed, topk=6, score_func="sigmoid", route_scale=2.5,
                   bias_std=0.01):
    from dsmoe import synth
    gen = torch.Generator().manual_seed(seed)
    experts = [synth.make_expert(fmt, hidden, inter, gen) for _ in range(n_experts)]
    shared = synth.make_expert("fp8", hidden, inter, gen)
    router = synth.make_router(n_experts, hidden, gen, bias_std=bias_std)
    return dict(fmt=fmt, hidden=hidden, inter=inter, n_experts=n_experts, topk=topk, score_func=score_func,
                route_scale=route_scale, experts=experts, shared=shared, router=router)


def to_oracle_expert(ew):
    n = lambda t: t.cpu().numpy()
    return OM.QuantExpert(ew.fmt, n(ew.w1), n(ew.s1), n(ew.w3), n(ew.s3), n(ew.w2), n(ew.s2))


def to_oracle_layer(spec):
    r = spec["router"]
    return OM.MoELayer(r.wg.numpy(), r.bias.numpy(), [to_oracle_expert(e) for e in spec["experts"]],
                       to_oracle_expert(spec["shared"]), spec["topk"], spec["score_func"], spec["route_scale"],
                       None if r.bias_vl is None else r.bias_vl.numpy())


def to_gpu_moe(spec, rank=0, world=1, device="cuda"):
    from dsmoe import MoE
    m = MoE(spec["hidden"], spec["inter"], spec["n_experts"], spec["topk"], spec["fmt"], spec["score_func"],
            spec["route_scale"], rank=rank, world=world, device=device)
    m.load_router(spec["router"])
    m.load_shared(spec["shared"])
    for e, ew in enumerate(spec["experts"]):
        m.load_expert(e, ew)
    return m


def bf16_np(x: torch.Tensor) -> np.ndarray:
    return x.float().cpu().numpy()
