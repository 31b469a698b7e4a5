"""The oracle (numpy restatement) against golden vectors made by the reference's own CPU code.

The fixtures come from tests/golden/make_golden.py (the reference's kernel.py shim, its fp4lib.c and
the torch lines of dsv41/tt/moe.py). These tests need no GPU.
"""
import numpy as np
import pytest

from oracle import formats as F
from oracle import moe as M
from oracle import ref_fp4lib


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_fp4_unpack_bit_exact(golden):
    out = F.dequant_fp4(golden["fp4deq_q"], golden["fp4deq_s"])
    assert np.array_equal(bits(out), bits(golden["fp4deq_out"]))          # shim, bit for bit
    assert np.array_equal(out, golden["fp4deq_out_c"])                    # fp4lib, value for value


@pytest.mark.skipif(not ref_fp4lib.available(), reason="reference fp4lib not built / no AVX-512")
def test_fp4_unpack_vs_reference_c():
    rng = np.random.default_rng(5)
    q = rng.integers(0, 256, (64, 160), dtype=np.uint8)
    s = rng.integers(0, 255, (64, 10), dtype=np.uint8)
    assert np.array_equal(F.dequant_fp4(q, s), ref_fp4lib.dequant_fp4(q, s))


def test_fp8_block_dequant_bit_exact(golden):
    out = F.dequant_fp8_block(golden["fp8deq_b"], golden["fp8deq_s"])
    assert np.array_equal(bits(out), bits(golden["fp8deq_out"]))


def test_e4m3_table_matches_torch():
    import torch
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(bits(F.E4M3_TABLE), bits(ref)) or np.array_equal(
        np.isnan(F.E4M3_TABLE), np.isnan(ref)) and np.array_equal(
        F.E4M3_TABLE[~np.isnan(ref)], ref[~np.isnan(ref)])


def test_fp8_quantizer_bit_exact(golden):
    q, s = F.quant_fp8_block(golden["fp8q_w"])
    assert np.array_equal(bits(s), bits(golden["fp8q_s"]))
    assert np.array_equal(q, golden["fp8q_q"])


def test_fp4_quantizer_bit_exact(golden):
    q, s = F.quant_fp4_e8m0(golden["fp4q_w"])
    assert np.array_equal(s, golden["fp4q_s"])
    assert np.array_equal(q, golden["fp4q_q"])


def test_act_quant_modes(golden):
    x = golden["actq_x"]
    # FAKEQUANT=0: identity in fp32 with unit scales
    assert np.array_equal(golden["actq_off"], x)
    assert np.all(golden["actq_off_s"] == 1.0)
    # FAKEQUANT=1: e4m3 per 128 with scale amax/448 (or its power-of-two ceiling)
    for key, pow2 in (("actq_on", False), ("actq_pow2", True)):
        xb = x.reshape(x.shape[0], -1, 128)
        amax = np.maximum(np.abs(xb).max(-1, keepdims=True), np.float32(1e-4))
        s = (amax / np.float32(448.0)).astype(np.float32)
        if pow2:
            s = F.pow2_ceil(s)
        q = F.e4m3_encode(np.clip(xb / s, -448, 448)).reshape(x.shape)
        assert np.array_equal(s[..., 0], golden[key + "_s"])
        assert np.array_equal(q, golden[key])


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_gemm_vs_shim(golden, fmt):
    x = golden["gemm_x"]
    if fmt == "fp8":
        w = F.dequant_fp8_block(golden["gemm_q8"], golden["gemm_s8"])
    else:
        w = F.dequant_fp4(golden["gemm_q4"], golden["gemm_s4"])
    y = F.bf16_round((x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32))
    ref = golden["gemm_y" + fmt[-1]]
    # the shim sums in fp32 (BLAS order) before its bf16 rounding: allow one bf16 ulp
    assert np.all(np.abs(y - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-30)


@pytest.mark.parametrize("sf,rs", [("sigmoid", 2.5), ("sqrtsoftplus", 1.5)])
def test_router_vs_reference(golden, sf, rs):
    x, wg, bias = golden["rt_x"], golden["rt_wg"], golden["rt_bias"]
    logits = M.router_logits(x, wg)
    # fp64-accumulated logits vs the Gate's fp32 matmul: same to fp32 rounding noise
    assert np.allclose(logits, golden["rt_logits"], rtol=1e-5, atol=1e-6)
    idx, wt, sc = M.route(x, wg, bias, 6, sf, rs)
    assert np.array_equal(idx, golden[f"rt_{sf}_idx"])
    assert np.allclose(wt, golden[f"rt_{sf}_wt"], rtol=1e-5, atol=0)
    assert np.allclose(sc, golden[f"rt_{sf}_sc"], rtol=1e-5, atol=1e-7)


def _layer_from_golden(golden, fmt):
    pre = f"moe_{fmt}_"
    n_exp = golden[pre + "wg"].shape[0]

    def ex(j, f):
        g = lambda nm: golden[f"{pre}e{j}_{nm}"]
        return M.QuantExpert(f, g("w1"), g("s1"), g("w3"), g("s3"), g("w2"), g("s2"))

    return M.MoELayer(golden[pre + "wg"], golden[pre + "bias"],
                      [ex(j, fmt) for j in range(n_exp)], ex(n_exp, "fp8"))


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_moe_layer_vs_reference(golden, fmt):
    pre = f"moe_{fmt}_"
    layer = _layer_from_golden(golden, fmt)
    x = golden[pre + "x"]
    for mimic in (False, True):
        y, idx, wt = M.moe_forward(layer, x, mimic_bf16=mimic)
        assert np.array_equal(idx, golden[pre + "idx"])
        assert np.allclose(wt, golden[pre + "wt"], rtol=1e-5)
        mar, cos = M.compare(y, golden[pre + "y"])
        assert mar < 1e-2 and cos > 0.9999, (mimic, mar, cos)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_partials_sum_to_full(golden, world):
    layer = _layer_from_golden(golden, "fp4")
    x = golden["moe_fp4_x"]
    full, _, _ = M.moe_forward(layer, x, return_partial=True)
    parts = sum(M.moe_forward(layer, x, r, world, return_partial=True)[0] for r in range(world))
    assert np.allclose(parts, full, rtol=1e-9, atol=1e-12)
