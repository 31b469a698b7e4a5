"""Writes tests/golden/*.npz: golden vectors produced by the REFERENCE's own CPU code.

Run in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_golden.py [--ref PATH]

PATH is the reference checkout: by default the DSV41_REFERENCE environment variable, else a
directory named ``reference`` beside this repository.

What runs:
* ``dsv41/ref/kernel.py`` -- the reference's plain-PyTorch operator shim -- imported from the
  reference checkout with ``DSV41_FAKEQUANT=0`` (dsv41/ref/kernel.py:36-47), plus a second copy
  with fake-quant on for ``act_quant``'s quantizing branch;
* ``dsv41/ref/fp4lib.c`` compiled unmodified by oracle/Makefile (oracle/_ref/libfp4.so);
* the router and expert-FFN steps of ``dsv41/tt/moe.py`` (it imports ttnn, so its torch lines
  -- moe.py:121-125 for the router, moe.py:133-139 for the FFN -- are executed here as written
  there, on CPU tensors, with every linear going through the shim's fp8_gemm / fp4_gemm under
  bf16 default dtype, dsv41/ref/load.py:38).

The fixtures are small (about 1 MB compressed) and seeded.
"""
import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def load_kernel(ref: str, fakequant: bool):
    os.environ["DSV41_FAKEQUANT"] = "1" if fakequant else "0"
    path = os.path.join(ref, "dsv41", "ref", "kernel.py")
    spec = importlib.util.spec_from_file_location(f"ref_kernel_fq{int(fakequant)}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.FAKEQUANT == fakequant
    return mod


def u8(t):
    return t.contiguous().view(torch.uint8).numpy().copy()


def fp8_quant_torch(w: torch.Tensor):
    """Benchmark-configuration FP8 generator: scale = blockmax/448 per 128x128, e4m3 cast."""
    n, k = w.shape
    nb, kb = -(-n // 128), -(-k // 128)
    pad = torch.zeros(nb * 128, kb * 128)
    pad[:n, :k] = w
    s = pad.abs().unflatten(0, (nb, 128)).unflatten(-1, (kb, 128)).amax(dim=(1, 3)).clamp(min=1e-30) / 448.0
    srep = s.repeat_interleave(128, 0)[:n].repeat_interleave(128, 1)[:, :k]
    q = (w / srep).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q, s


def fp4_quant_torch(K, w: torch.Tensor):
    """Benchmark-configuration FP4 generator from the shim's own helpers (kernel.py:15-29, 69-70)."""
    n, k = w.shape
    wb = w.unflatten(-1, (-1, 32))
    amax = wb.abs().amax(-1, keepdim=True)
    s = K._pow2_ceil(amax.clamp(min=6 * 2.0 ** -126) / 6.0)
    v = K._to_fp4(wb / s).flatten(-2)
    grid = K.FP4_GRID
    mag = (v.abs().unsqueeze(-1) == grid).float().argmax(-1).to(torch.uint8)
    code = mag | (((v < 0) & (mag > 0)).to(torch.uint8) << 3)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    e8 = s.squeeze(-1).to(torch.float8_e8m0fnu)
    return packed.contiguous(), e8.contiguous()


def make_expert(K, fmt, H, I, gen):
    ws = {nm: torch.randn(shape, generator=gen) * 0.02
          for nm, shape in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I)))}
    out = {}
    for nm, w in ws.items():
        if fmt == "fp8":
            q, s = fp8_quant_torch(w)
        else:
            q, s = fp4_quant_torch(K, w)
        out[nm] = (q, s)
    return out


def ref_linear(K, fmt, x_bf16, q, s):
    """One linear through the shim with FAKEQUANT off: act_quant -> fp8_gemm / fp4_gemm."""
    a, a_s = K.act_quant(x_bf16, 128)
    if fmt == "fp8":
        return K.fp8_gemm(a, a_s, q, s)
    return K.fp4_gemm(a, a_s, q, s)


def ref_ffn(K, fmt, x, e, wt=None):
    """dsv41/tt/moe.py:133-139 with torch ops and shim linears (bf16 outputs)."""
    LIMIT = 10.0
    g = ref_linear(K, fmt, x, *e["w1"]).clamp(max=LIMIT)
    u = ref_linear(K, fmt, x, *e["w3"]).clamp(min=-LIMIT, max=LIMIT)
    h = torch.nn.functional.silu(g) * u
    if wt is not None:
        h = h * wt.to(h.dtype).unsqueeze(-1)
    return ref_linear(K, fmt, h, *e["w2"])


def ref_route(logits, bias, topk, score_func, route_scale):
    """dsv41/tt/moe.py:121-125 (score function chosen by the configuration)."""
    if score_func == "sqrtsoftplus":
        sc = torch.nn.functional.softplus(logits.float()).sqrt()
    else:
        sc = torch.sigmoid(logits.float())
    idx = (sc + bias).topk(topk, dim=-1).indices
    wt = sc.gather(1, idx)
    return idx, wt / (wt.sum(-1, keepdim=True) + 1e-20) * route_scale, sc


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DSV41_REFERENCE")
                    or os.path.join(os.path.dirname(ROOT), "reference"))
    args = ap.parse_args()
    K = load_kernel(args.ref, fakequant=False)
    KQ = load_kernel(args.ref, fakequant=True)
    from oracle import ref_fp4lib

    torch.set_default_dtype(torch.float32)
    gen = torch.Generator().manual_seed(1234)
    fx = {}

    # 1. FP4 unpack: random bytes, scales over a wide range incl. the extremes 0 and 254.
    q = torch.randint(0, 256, (48, 64), generator=gen, dtype=torch.uint8)
    s = torch.randint(100, 150, (48, 4), generator=gen, dtype=torch.uint8)
    s[0, 0], s[1, 1], s[2, 2], s[3, 3] = 0, 1, 127, 254
    out_t = K.dequant_fp4_weight(q, s.view(torch.float8_e8m0fnu))
    out_c = ref_fp4lib.dequant_fp4(q.numpy(), s.numpy())
    # The two reference paths agree on every value; they differ only in the sign of zero for
    # nibble 8 (-0.0 from the shim's table, +0.0 from fp4lib's integer LUT). Bits are pinned to
    # the shim (the documented operator), values to both.
    assert np.array_equal(out_t.numpy(), out_c), "shim vs fp4lib values"
    fx.update(fp4deq_q=q.numpy(), fp4deq_s=s.numpy(), fp4deq_out=out_t.numpy(), fp4deq_out_c=out_c)

    # 2. FP8 block dequant, ragged shape (not a multiple of 128), no NaN codes.
    b = torch.randint(0, 256, (200, 300), generator=gen, dtype=torch.uint8)
    b[(b & 0x7F) == 0x7F] = 0x42
    bs = torch.rand((2, 3), generator=gen) * 1e-3 + 1e-5
    out = K._deq_fp8_weight(b.view(torch.float8_e4m3fn), bs, 128)
    fx.update(fp8deq_b=b.numpy(), fp8deq_s=bs.numpy(), fp8deq_out=out.numpy())

    # 3. quantizers (the configuration's weight generators)
    w8 = torch.randn((200, 300), generator=gen) * 0.02
    q8, s8 = fp8_quant_torch(w8)
    fx.update(fp8q_w=w8.numpy(), fp8q_q=u8(q8), fp8q_s=s8.numpy())
    w4 = torch.randn((64, 256), generator=gen) * 0.02
    w4[0, :32] = 0.0                                         # an all-zero group
    q4, s4 = fp4_quant_torch(K, w4)
    fx.update(fp4q_w=w4.numpy(), fp4q_q=q4.numpy(), fp4q_s=u8(s4))

    # 4. act_quant in both modes (kernel.py:44-55)
    xa = (torch.randn((3, 256), generator=gen) * 3).to(torch.bfloat16)
    a0, a0s = K.act_quant(xa, 128)
    a1, a1s = KQ.act_quant(xa, 128)
    a2, a2s = KQ.act_quant(xa, 128, scale_fmt="ue8m0")
    fx.update(actq_x=xa.float().numpy(), actq_off=a0.numpy(), actq_off_s=a0s.numpy(),
              actq_on=u8(a1), actq_on_s=a1s.numpy(), actq_pow2=u8(a2), actq_pow2_s=a2s.numpy())

    # 5./6. fp8_gemm and fp4_gemm (bf16 default dtype, as the model sets it)
    torch.set_default_dtype(torch.bfloat16)
    x = torch.randn((3, 512), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    wq = torch.randn((256, 512), generator=gen, dtype=torch.float32) * 0.02
    q8g, s8g = fp8_quant_torch(wq)
    q4g, s4g = fp4_quant_torch(K, wq)
    a, a_s = K.act_quant(x, 128)
    y8 = K.fp8_gemm(a, a_s, q8g, s8g)
    y4 = K.fp4_gemm(a, a_s, q4g, s4g)
    assert y8.dtype == torch.bfloat16 and y4.dtype == torch.bfloat16
    fx.update(gemm_x=x.float().numpy(), gemm_q8=u8(q8g), gemm_s8=s8g.float().numpy(),
              gemm_q4=q4g.numpy(), gemm_s4=u8(s4g), gemm_y8=y8.float().numpy(), gemm_y4=y4.float().numpy())
    torch.set_default_dtype(torch.float32)

    # 7. router (moe.py:108-125): fp32 logits as the Gate computes them
    H, E = 512, 64
    xr = torch.randn((16, H), generator=gen).to(torch.bfloat16)
    wg = torch.randn((E, H), generator=gen) * 0.02
    bias = torch.randn((E,), generator=gen) * 0.01
    logits = xr.float() @ wg.T
    fx.update(rt_x=xr.float().numpy(), rt_wg=wg.numpy(), rt_bias=bias.numpy(), rt_logits=logits.numpy())
    for sf, rs in (("sigmoid", 2.5), ("sqrtsoftplus", 1.5)):
        idx, wt, sc = ref_route(logits, bias, 6, sf, rs)
        fx[f"rt_{sf}_idx"] = idx.numpy()
        fx[f"rt_{sf}_wt"] = wt.numpy()
        fx[f"rt_{sf}_sc"] = sc.numpy()

    # 8. one small MoE layer per format: E routed + 1 shared, top-6, B tokens; shared stays FP8
    torch.set_default_dtype(torch.bfloat16)
    H, I, E, B = 256, 128, 8, 4
    for fmt in ("fp8", "fp4"):
        g2 = torch.Generator().manual_seed(77 if fmt == "fp8" else 78)
        experts = [make_expert(K, fmt, H, I, g2) for _ in range(E)]
        shared = make_expert(K, "fp8", H, I, g2)
        wgl = torch.randn((E, H), generator=g2, dtype=torch.float32) * 0.02
        bl = torch.randn((E,), generator=g2, dtype=torch.float32) * 0.01
        xl = torch.randn((B, H), generator=g2, dtype=torch.float32).to(torch.bfloat16)
        idx, wt, _ = ref_route(xl.float() @ wgl.T, bl, 6, "sigmoid", 2.5)
        y = ref_ffn(K, "fp8", xl, shared).float()
        for e in idx.unique().tolist():
            tok, kk = torch.where(idx == e)
            y[tok] += ref_ffn(K, fmt, xl[tok], experts[e], wt[tok, kk]).float()
        pre = f"moe_{fmt}_"
        fx.update({pre + "x": xl.float().numpy(), pre + "wg": wgl.numpy(), pre + "bias": bl.numpy(),
                   pre + "idx": idx.numpy(), pre + "wt": wt.float().numpy(),
                   pre + "y": y.to(torch.bfloat16).float().numpy()})
        for j, ex in enumerate(experts + [shared]):
            f = fmt if j < E else "fp8"
            for nm in ("w1", "w3", "w2"):
                qq, ss = ex[nm]
                fx[f"{pre}e{j}_{nm}"] = u8(qq)
                fx[f"{pre}e{j}_s{nm[1:]}"] = ss.float().numpy() if f == "fp8" else u8(ss)
    torch.set_default_dtype(torch.float32)

    path = os.path.join(HERE, "golden_ref.npz")
    np.savez_compressed(path, **fx)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(fx)} arrays)")


if __name__ == "__main__":
    main()
