"""The kernel-surface GEMMs (dsmoe_fp8_gemm / dsmoe_fp4_gemm: fp8_gemm / fp4_gemm of
dsv41/ref/kernel.py:105-112) on the tcgen05 path, against a float64 restatement of the same op:
out = (a * a_s per 128-K block) @ dequant(b, b_s)^T.

Shapes cover one and several token tiles (16 / 32 / 64 / 128 tokens per tile, ragged M), ragged N (rows
past the last 128-row tile), split K (few tiles: partials summed by the last CTA of each tile) and
whole-tile launches; activations in fp32, bf16 and e4m3 with and without per-block scales; fp32 and
bf16 outputs. Bars: weights enter exactly, each scaled activation is carried as bf16 hi + lo
(relative error <= 2^-17), products accumulate in fp32, so |out - ref| <= 4e-5 * sum|a_k w_k| (plus
one bf16 rounding of the result for bf16 outputs). Repeated calls give the same bits."""
import numpy as np
import pytest
import torch

from oracle import formats as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import dsmoe  # noqa: F401
    return torch.device("cuda", 0)


def _weights(fmt, N, K, rng):
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    if fmt == "fp8":
        q, s = F.quant_fp8_block(w)
        return q, s, F.dequant_fp8_block(q, s).astype(np.float64)
    q, s = F.quant_fp4_e8m0(w)
    return q, s, F.dequant_fp4(q, s).astype(np.float64)


def _acts(adt, M, K, scaled, rng):
    x = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    if adt == "e4m3":  # act_quant's fake-quant form: e4m3 codes + fp32 scale per 128-K block
        xb = x.reshape(M, K // 128, 128)
        sa = (np.maximum(np.abs(xb).max(-1), 1e-4) / 448.0).astype(np.float32)
        codes = F.e4m3_encode(np.clip(xb / sa[..., None], -448, 448)).reshape(M, K)
        vals = F.e4m3_decode(codes).astype(np.float64)
        return codes, (sa if scaled else None), vals
    if adt == "bf16":
        x = F.bf16_round(x)
    sa = (rng.uniform(0.5, 2.0, (M, K // 128))).astype(np.float32) if scaled else None
    return x, sa, x.astype(np.float64)


def _run(dev, fmt, adt, M, N, K, scaled, out_f32, seed):
    from dsmoe import _lib as L
    rng = np.random.default_rng(seed)
    q, s, wd = _weights(fmt, N, K, rng)
    xa, sa, xv = _acts(adt, M, K, scaled, rng)
    av = xv * (np.repeat(sa, 128, axis=1).astype(np.float64) if sa is not None else 1.0)
    ref = av @ wd.T
    bound = np.abs(av) @ np.abs(wd).T
    if adt == "e4m3":
        at, code = torch.from_numpy(xa).to(dev), L.DTYPE_E4M3
    elif adt == "bf16":
        at, code = torch.from_numpy(xa).to(torch.bfloat16).to(dev), L.DTYPE_BF16
    else:
        at, code = torch.from_numpy(xa).to(dev), L.DTYPE_F32
    ast = torch.from_numpy(sa).to(dev) if sa is not None else None
    bt, bst = torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev)
    out = torch.empty((M, N), dtype=torch.float32 if out_f32 else torch.bfloat16, device=dev)
    fn = "dsmoe_fp8_gemm" if fmt == "fp8" else "dsmoe_fp4_gemm"
    args = (L.ptr(at), code, L.ptr(ast), M, K, L.ptr(bt), L.ptr(bst), N, L.ptr(out),
            L.DTYPE_F32 if out_f32 else L.DTYPE_BF16, L.stream_of(at))
    L.call(fn, *args)
    y = out.float().cpu().numpy().astype(np.float64)
    out2 = out.clone()
    L.call(fn, *args)
    assert torch.equal(out, out2), "repeated calls differ"
    tol = 4e-5 * bound + 1e-30
    if not out_f32:
        tol = tol + np.abs(ref) * 2.0 ** -8
    err = np.abs(y - ref)
    assert np.isfinite(y).all()
    assert np.all(err <= tol), (fmt, adt, M, N, K, float((err / np.maximum(tol, 1e-30)).max()))


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("M,N,K", [(1, 256, 1024), (5, 384, 512), (16, 128, 128), (17, 200, 384),
                                   (33, 1000, 256), (64, 256, 640), (130, 384, 256), (300, 128, 384)])
def test_gemm_shapes_f32(dev, fmt, M, N, K):
    _run(dev, fmt, "f32", M, N, K, True, True, seed=M * 7 + N + K)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("adt", ["f32", "bf16", "e4m3"])
@pytest.mark.parametrize("scaled", [True, False])
@pytest.mark.parametrize("out_f32", [True, False])
def test_gemm_dtypes(dev, fmt, adt, scaled, out_f32):
    seed = 100 + 8 * ["f32", "bf16", "e4m3"].index(adt) + 4 * (fmt == "fp4") + 2 * scaled + out_f32
    _run(dev, fmt, adt, 9, 256, 512, scaled, out_f32, seed=seed)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
@pytest.mark.parametrize("M,N,K", [(1, 384, 640), (20, 384, 640), (40, 256, 512), (65, 384, 640), (100, 1000, 384),
                                   (300, 1000, 384), (600, 7680, 256)])
def test_gemm_e4m3_tiles(dev, fmt, M, N, K):
    """FP8 / FP4 weights x e4m3 activations (the no-conversion kernel; FP4 through the block-scaled
    MMA): 16 / 32 / 64 / 128 tokens per tile, split and unsplit K, ragged M and N."""
    _run(dev, fmt, "e4m3", M, N, K, True, False, seed=M + N + K + (fmt == "fp4"))


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_gemm_split_k_large_k(dev, fmt):
    """One token over a 5120-wide K: 40 K blocks split over several CTAs per tile."""
    _run(dev, fmt, "e4m3", 1, 512, 5120, True, False, seed=51)


@pytest.mark.parametrize("fmt", ["fp8", "fp4"])
def test_gemm_many_tiles(dev, fmt):
    """More tiles than SMs (no split): 3 token tiles x 60 row tiles."""
    _run(dev, fmt, "bf16", 150, 7680, 256, True, False, seed=77)


def test_gemm_rejects_bad_arguments(dev):
    from dsmoe import _lib as L
    x = torch.zeros((4, 256), dtype=torch.float32, device=dev)
    b = torch.zeros((128, 256), dtype=torch.uint8, device=dev)
    s = torch.ones((1, 2), dtype=torch.float32, device=dev)
    out = torch.empty((4, 128), dtype=torch.float32, device=dev)
    st = L.stream_of(x)
    assert L.lib.dsmoe_fp8_gemm(L.ptr(x), L.DTYPE_F32, None, 4, 200, L.ptr(b), L.ptr(s), 128, L.ptr(out),
                                L.DTYPE_F32, st) == L.ERR_ARG  # K not a multiple of 128
    assert L.lib.dsmoe_fp8_gemm(L.ptr(x) + 4, L.DTYPE_F32, None, 4, 128, L.ptr(b), L.ptr(s), 128, L.ptr(out),
                                L.DTYPE_F32, st) == L.ERR_ALIGN  # activations not 16-byte aligned
