"""NVFP4 number formats and the per-expert dequantisation, restated in numpy (test infrastructure only).

Follows bench/moek/problem.py:17-38 (the reference's E2M1 table, nibble order and ``dequant``): a checkpoint expert
is ``weight`` uint8 [N, K/2] (element 2i in the low nibble, 2i+1 in the high nibble), ``weight_scale`` float8 E4M3
[N, K/16] (one per 16 inputs along K) and ``weight_scale_2`` fp32 (one per expert). The dequantised weight is
``e2m1(code) * float(scale) * gs`` computed in fp32 and rounded to bf16 (problem.py:36-38).
"""
import numpy as np

# E2M1 code -> value; bit 3 is the sign (bench/moek/problem.py:17)
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                 -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e4m3_table() -> np.ndarray:
    """float8 E4M3 (fn variant: no infinities, 0x7F/0xFF are NaN) bit pattern -> fp32 value, from the format."""
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 15 and m == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = e4m3_table()


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, on the bit patterns (NaN kept as NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def dequant_expert(codes: np.ndarray, scales_u8: np.ndarray, gs: float) -> np.ndarray:
    """One expert to bf16-valued fp32 [N, K] (bench/moek/problem.py:31-38).

    codes: uint8 [N, K/2]; scales_u8: the E4M3 bit patterns [N, K/16]; gs: the expert's fp32 weight_scale_2.
    """
    lo = E2M1[codes & 0xF]
    hi = E2M1[codes >> 4]
    v = np.stack([lo, hi], -1).reshape(codes.shape[0], -1)  # [N, K], element 2i from the low nibble
    sc = np.repeat(E4M3[scales_u8], 16, axis=1)
    return bf16_round(v * sc * np.float32(gs))
