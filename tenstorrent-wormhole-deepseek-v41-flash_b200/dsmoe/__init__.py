"""dsmoe -- B200-native quantized MoE expert layer (host side).

The compute lives in libdsmoe.so (CUDA, sm_100a) behind the C ABI in include/dsmoe.h; this package
binds it (``_lib``), keeps the resident expert store (``store``), and exposes the reference's
Gate / Expert / MoE surface (``moe``), and replays the decode calls of a set of layers as one CUDA
graph (``trace``, the reference's traced decode step). Synthetic seeded weights for tests and benchmarks are in
``synth``.
"""
from . import _lib
from .moe import MoE, Gate, Expert
from .store import ExpertStore, expert_bytes
from .trace import DecodeTrace
from .synth import ExpertWeights, RouterWeights, make_expert, make_router, make_tokens, zipf_routing

__all__ = ["MoE", "Gate", "Expert", "DecodeTrace", "ExpertStore", "expert_bytes", "ExpertWeights", "RouterWeights",
           "make_expert", "make_router", "make_tokens", "zipf_routing", "_lib"]
