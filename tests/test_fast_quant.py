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


def test_packed_screen_range_flags_match_the_per_half_rule():
    """The screened router checks both BF16 halves of a word at once
    (ninfer_nvfp4_glm-5.3_flash_2x_dgxspark_b200/csrc/nf_kernels.cu
    bf16x2_screen_flags): with m the 15-bit magnitudes per 16-bit lane,
    bit 15 of (m + 0x3680) | (~(m + 0x6200) & (m + 0x7fff)) is set exactly
    when the half is nonzero with its exponent field below 60 or above 146
    (the scalar rule, bf16_screen_unsafe).  Checked for every low half with
    random high halves and every high half with random low halves (no carry
    may cross the lanes)."""
    def flags(u):
        m = u & np.uint64(0x7FFF7FFF)
        hi = (m + np.uint64(0x36803680)) & np.uint64(0xFFFFFFFF)
        lo = (~((m + np.uint64(0x62006200)) & np.uint64(0xFFFFFFFF))) & ((m + np.uint64(0x7FFF7FFF)) & np.uint64(0xFFFFFFFF))
        return (hi | lo) & np.uint64(0x80008000)

    def rule(h):
        e = (h >> np.uint64(7)) & np.uint64(0xFF)
        return ((h & np.uint64(0x7FFF)) != 0) & ((e < 60) | (e > 146))

    halves = np.arange(65536, dtype=np.uint64)
    rng = np.random.Generator(np.random.PCG64(3))
    for _ in range(4):
        other = rng.integers(0, 65536, 65536).astype(np.uint64)
        f = flags(halves | (other << np.uint64(16)))
        assert np.array_equal((f & np.uint64(0x8000)) != 0, rule(halves))
        assert np.array_equal((f & np.uint64(0x80000000)) != 0, rule(other))
        f = flags(other | (halves << np.uint64(16)))
        assert np.array_equal((f & np.uint64(0x80000000)) != 0, rule(halves))
        assert np.array_equal((f & np.uint64(0x8000)) != 0, rule(other))
