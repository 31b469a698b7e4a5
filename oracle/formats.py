"""Weight formats of the MoE path, restated in numpy (oracle; test infrastructure only).

FP8 e4m3 ("e4m3fn": no infinities, 0x7F/0xFF are NaN) with fp32 scales per 128x128 block, and
FP4 e2m1 packed two per byte (LOW nibble first, bit 3 = sign) with one e8m0 scale per 32
consecutive K elements.

Each function cites the reference line it follows.
"""
import numpy as np

# e2m1 magnitudes by 3-bit code; bit 3 of the nibble is the sign (dsv41/ref/kernel.py:10-12,
# dsv41/ckpt.py:13).
FP4_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
FP4_TABLE = np.concatenate([FP4_GRID, -FP4_GRID]).astype(np.float32)

E4M3_MAX = 448.0


def _e4m3_decode_table() -> np.ndarray:
    """All 256 e4m3fn codes -> float32.

    Bias 7, subnormals m/8 * 2^-6. 0x7F and 0xFF decode to NaN, which is what
    ``b.float()`` does in the reference dequant (dsv41/ref/kernel.py:75-78, torch float8_e4m3fn).
    The Tenstorrent loader's LUT maps those two codes to 0.0 instead (dsv41/tt/weights.py:16-22);
    quantized weights never contain them.
    """
    t = np.empty(256, dtype=np.float32)
    for b in range(256):
        s, e, m = b >> 7, (b >> 3) & 0xF, b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
            continue
        v = (m / 8.0) * 2.0 ** -6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[b] = -v if s else v
    return t


E4M3_TABLE = _e4m3_decode_table()
# positive finite codes 0..126 are monotonic in value
_E4M3_POS = E4M3_TABLE[:127].astype(np.float64)


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float -> e4m3fn code, round to nearest, ties to the even code; |x| must be <= 448.

    This is the cast ``(w / s).clamp(-448, 448).to(torch.float8_e4m3fn)`` used to make FP8 weights
    (the same cast as dsv41/ref/kernel.py:51). A negative value keeps its sign bit even when it
    rounds to zero (0x80), as the torch cast does.
    """
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), E4M3_MAX)
    hi = np.searchsorted(_E4M3_POS, a, side="left").clip(max=126)
    lo = np.maximum(hi - 1, 0)
    dlo = a - _E4M3_POS[lo]
    dhi = _E4M3_POS[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return code | (np.signbit(x).astype(np.uint8) << 7)


def pow2_ceil(x: np.ndarray) -> np.ndarray:
    """2**ceil(log2(x)) exactly, via frexp (dsv41/ref/kernel.py:15-18)."""
    m, e = np.frexp(np.asarray(x, dtype=np.float32))
    return np.ldexp(np.float32(1.0), np.where(m == 0.5, e - 1, e)).astype(np.float32)


def to_fp4_codes(x: np.ndarray) -> np.ndarray:
    """Round to the e2m1 grid, ties to the even code (dsv41/ref/kernel.py:21-29) -> 4-bit codes.

    A value that rounds to zero is coded +0 (code 0) whatever its sign.
    """
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x), np.float32(6.0))
    hi = np.searchsorted(FP4_GRID, a, side="left").clip(max=7)
    lo = np.maximum(hi - 1, 0)
    dlo = a - FP4_GRID[lo]
    dhi = FP4_GRID[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    mag = np.where(pick_hi, hi, lo).astype(np.uint8)
    neg = (x < 0) & (mag > 0)
    return mag | (neg.astype(np.uint8) << 3)


def e8m0_decode(b: np.ndarray) -> np.ndarray:
    """e8m0 byte -> 2^(b-127) as float32; 0xFF is NaN (torch float8_e8m0fnu, dsv41/ref/kernel.py:98)."""
    b = np.asarray(b, dtype=np.uint8)
    v = np.ldexp(np.float32(1.0), b.astype(np.int32) - 127).astype(np.float32)
    return np.where(b == 0xFF, np.float32(np.nan), v).astype(np.float32)


# ---------------------------------------------------------------- quantizers (synthetic weights)

def quant_fp8_block(w: np.ndarray, block: int = 128):
    """fp32 [N, K] -> (e4m3 codes [N, K] uint8, fp32 scales [ceil(N/b), ceil(K/b)]).

    scale = blockmax / 448 per block, q = e4m3(clamp(w / scale, +-448)). This is the generator the
    benchmark configuration prescribes for FP8 expert weights; the dequant that reads it back is
    dsv41/ref/kernel.py:75-78.
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    nb, kb = -(-n // block), -(-k // block)
    pad = np.zeros((nb * block, kb * block), dtype=np.float32)
    pad[:n, :k] = w
    blk = np.abs(pad).reshape(nb, block, kb, block).max(axis=(1, 3))
    s = (np.maximum(blk, np.float32(1e-30)) / np.float32(E4M3_MAX)).astype(np.float32)
    srep = np.repeat(np.repeat(s, block, 0), block, 1)[:n, :k]
    q = e4m3_encode(np.clip(w / srep, -E4M3_MAX, E4M3_MAX))
    return q, s


def quant_fp4_e8m0(w: np.ndarray, group: int = 32):
    """fp32 [N, K] -> (packed e2m1 [N, K/2] uint8, low nibble first; e8m0 scales [N, K/32] uint8).

    scale = pow2_ceil(max(amax, 6*2^-126) / 6) per 32 consecutive K values, codes = to_fp4(w / scale)
    (dsv41/ref/kernel.py:15-29, 69-70); packing follows dsv41/ckpt.py:5-6 (low nibble first).
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % group == 0 and k % 2 == 0
    wb = w.reshape(n, k // group, group)
    amax = np.abs(wb).max(axis=-1, keepdims=True)
    s = pow2_ceil(np.maximum(amax, np.float32(6 * 2.0 ** -126)) / np.float32(6.0))
    codes = to_fp4_codes(wb / s).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    e = (np.frexp(s)[1] - 1 + 127).astype(np.int32).reshape(n, k // group)
    return packed, e.astype(np.uint8)


# ---------------------------------------------------------------- dequant (the unpack oracle)

def dequant_fp8_block(b: np.ndarray, b_s: np.ndarray, block: int = 128) -> np.ndarray:
    """e4m3 codes [N, K] + fp32 scales [ceil(N/b), ceil(K/b)] -> fp32 [N, K] (dsv41/ref/kernel.py:75-78)."""
    n, k = b.shape
    s = np.repeat(np.asarray(b_s, np.float32), block, 0)[:n]
    s = np.repeat(s, block, 1)[:, :k]
    return (e4m3_decode(b) * s).astype(np.float32)


def dequant_fp4(b: np.ndarray, b_s: np.ndarray) -> np.ndarray:
    """packed e2m1 [N, K/2] (low nibble first) + e8m0 [N, K/32] -> fp32 [N, K].

    dsv41/ref/kernel.py:91-98 (torch LUT path) and dsv41/ref/fp4lib.c:12-30 (C path): value =
    FP4_TABLE[nibble] * 2^(scale-127).
    """
    u = np.asarray(b, dtype=np.uint8)
    n, half = u.shape
    idx = np.stack([u & 0x0F, u >> 4], axis=-1).reshape(n, half * 2)
    with np.errstate(over="ignore"):         # scale 254 times 6 overflows to inf, as in torch
        return (FP4_TABLE[idx] * np.repeat(e8m0_decode(b_s), 32, axis=1)).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest, ties to even) and return it as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(u: np.ndarray) -> np.ndarray:
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
