"""The gate/up epilogue's quantiser divides the group peak by 6 with an FMA
correction (Markstein) instead of a division: that it equals the correctly
rounded quotient for every value it can see -- every finite non-negative
BF16 value -- is checked here exhaustively, with exact rational arithmetic
for each single-rounding step (ninfer_nvfp4_glm-5.3_flash_2x_dgxspark_b200/
csrc/nf_gemm_shared.cuh div6_rn)."""
import struct
from fractions import Fraction

import numpy as np


def f32_round(fr: Fraction) -> float:
    """fr rounded to the nearest fp32 value, ties to even."""
    if fr == 0:
        return 0.0
    sign = -1.0 if fr < 0 else 1.0
    a = abs(fr)
    x = np.float32(float(a))
    best = None
    for c in (x, np.nextafter(x, np.float32(np.inf)), np.nextafter(x, np.float32(0))):
        d = abs(Fraction(float(c)) - a)
        even = (struct.unpack("<I", struct.pack("<f", float(c)))[0] & 1) == 0
        if best is None or d < best[0] or (d == best[0] and even):
            best = (d, float(c))
    return sign * best[1]


def test_fma_corrected_division_by_six_is_exact_for_every_bf16_value():
    r6 = float(np.float32(1.0) / np.float32(6.0))
    assert struct.pack("<f", r6) == struct.pack("<f", 0.16666667163372039794921875)
    for bits in range(0, 0x7F80):  # +0 .. the largest finite BF16 value
        p = struct.unpack("<f", struct.pack("<I", bits << 16))[0]
        q = f32_round(Fraction(p) * Fraction(r6))
        r = f32_round(-Fraction(q) * 6 + Fraction(p))
        q2 = f32_round(Fraction(r) * Fraction(r6) + Fraction(q))
        assert q2 == f32_round(Fraction(p) / 6), hex(bits)
