"""CPU-only checks of the C ABI library and the host logic (no GPU calls)."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsmoe.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DSMOE_API\s+[\w\s\*]+?\b(dsmoe_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("dsmoe_moe_decode", "dsmoe_router", "dsmoe_store_pack_expert", "dsmoe_fp8_gemm",
              "dsmoe_fp4_gemm", "dsmoe_fp4_dequant", "dsmoe_fp8_block_dequant"):
        assert s in syms


def test_library_loads_and_exports_every_declared_symbol():
    from dsmoe import _lib as L
    raw = ctypes.CDLL(L.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(raw, s)]
    assert not missing, missing
    assert L.lib.dsmoe_version() >= 1


def test_every_header_symbol_has_a_python_signature():
    from dsmoe import _lib as L
    have = set(L._SIGS) | {"dsmoe_last_error"}
    assert set(declared_symbols()) <= have


def test_store_sizes_match_the_algorithmic_bytes():
    """FP4 store = exactly the algorithmic expert bytes; FP8 adds the per-tile scale copies (<0.4 %)."""
    from dsmoe import expert_bytes
    a, b = expert_bytes("fp4", 5120, 2048)
    assert a + b == 16_711_680
    a8, b8 = expert_bytes("fp8", 5120, 2048)
    alg = 3 * 5120 * 2048 + 3 * 16 * 40 * 4
    assert alg <= a8 + b8 <= alg * 1.004
    # tensor-parallel slices partition the store
    a1, b1 = expert_bytes("fp4", 5120, 256)
    assert 8 * (a1 + b1) == a + b


@pytest.mark.parametrize("fmt,H,I", [("fp8", 5120, 100), ("fp4", 5120, 96), ("fp8", 5000, 2048)])
def test_store_geometry_rejected(fmt, H, I):
    from dsmoe import expert_bytes, _lib as L
    with pytest.raises(L.DsmoeError) as ei:
        expert_bytes(fmt, H, I)
    assert ei.value.code == L.ERR_ARG


def test_entry_points_validate_before_touching_the_device():
    from dsmoe import _lib as L
    lay = L.Layer()
    lay.hidden, lay.inter_local, lay.n_experts, lay.topk = 5120, 2048, 384, 6
    assert L.lib.dsmoe_moe_workspace_bytes(ctypes.byref(lay), 8) > 0
    # null router weights -> ERR_ARG, no launch
    rc = L.lib.dsmoe_router(ctypes.byref(lay), None, 1, None, None, None, None, None, 0, None)
    assert rc == L.ERR_ARG and b"router" in L.lib.dsmoe_last_error()
    assert L.lib.dsmoe_fp4_dequant(None, None, 4, 64, None, L.DTYPE_F32, None) == L.ERR_ARG
    assert L.lib.dsmoe_fp8_gemm(None, 0, None, 1, 128, None, None, 1, None, 0, None) == L.ERR_ARG


def test_tp_slices():
    from dsmoe.tp import slice_of
    assert slice_of(2048, 3, 8) == (768, 256)
    assert slice_of(2304, 1, 8) == (288, 288)     # the real model's 2304 over 8 GPUs
    with pytest.raises(ValueError):
        slice_of(2304, 0, 16)                      # 144 rows: breaks the 32-row alignment
    with pytest.raises(ValueError):
        slice_of(2048, 0, 3)                       # uneven split
    assert slice_of(2048, 0, 1) == (0, 2048)


def test_slot_plan_rule_restated():
    """The decode slot plan (experts in id order, <= 8 tokens per slot, shared expert last),
    restated on the CPU: the number of slots for the benchmark's batches stays within the bound
    the workspace is sized for."""
    rng = np.random.default_rng(0)
    for B in (1, 4, 8, 64):
        idx = np.stack([rng.choice(384, 6, replace=False) for _ in range(B)])
        counts = np.bincount(idx.ravel(), minlength=384)
        slots = int(np.sum((counts + 7) // 8)) + (B + 7) // 8
        assert slots <= B * 6 + (B + 7) // 8


class _FakeLayer:
    """Just the attributes DecodeTrace checks before it touches a GPU."""

    def __init__(self, hidden=1024, world=1, comm=None, max_tokens=64, device="cuda:0"):
        self.hidden, self.world, self.comm, self.max_tokens, self.device = hidden, world, comm, max_tokens, device


def test_decode_trace_rejects_bad_layer_sets():
    from dsmoe import DecodeTrace
    with pytest.raises(ValueError):
        DecodeTrace([], 1)
    with pytest.raises(ValueError):  # one trace, one hidden size
        DecodeTrace([_FakeLayer(1024), _FakeLayer(2048)], 1)
    with pytest.raises(ValueError):  # one trace, one GPU
        DecodeTrace([_FakeLayer(device="cuda:0"), _FakeLayer(device="cuda:1")], 1)
    for bad in (0, 65):
        with pytest.raises(ValueError):
            DecodeTrace([_FakeLayer()], bad)
    with pytest.raises(ValueError):  # world > 1: the all-reduce must run inside the decode kernel
        DecodeTrace([_FakeLayer(world=2)], 1)
    with pytest.raises(ValueError):  # ... which takes at most 8 tokens
        DecodeTrace([_FakeLayer(world=2, comm=object())], 9)


def test_copy_async_rejects_null_arguments():
    from dsmoe import _lib as L
    assert L.lib.dsmoe_copy_async(None, None, 16, None) == L.ERR_ARG
    assert L.lib.dsmoe_copy_async(None, None, -1, None) == L.ERR_ARG
