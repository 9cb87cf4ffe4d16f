"""Pins the CPU oracle (and, when built, the reference's own sources) to the
known-answer values of the reference's tests:
  tests/test_nvfp4_decode.cpp:25-86, tests/test_nvfp4_view.cpp:14-137,
  tests/test_text_forward.cpp:311-370, tests/test_tiny_layer.cpp:21-46.
"""
import ctypes
import math
import struct

import numpy as np
import pytest

from helpers import oracle

orc = oracle()
P = orc.p


def libs():
    out = [("port", orc.port())]
    r = orc.ref()
    if r is not None:
        out.append(("ref", r))
    return out


def fn(lib, name):
    return getattr(lib, ("or_" if hasattr(lib, "or_e2m1") else "ref_") + name)


def independent_fp8(bits: int) -> float:
    """IEEE bit construction of E4M3FN (tests/test_nvfp4_view.cpp:14-21)."""
    exponent, mantissa = (bits >> 3) & 15, bits & 7
    if exponent == 15 and mantissa == 7:
        return math.nan
    if exponent == 0:
        mag = mantissa / 512.0
    else:
        mag = struct.unpack("<f", struct.pack("<I", ((exponent + 120) << 23) | (mantissa << 20)))[0]
    return -mag if bits & 128 else mag


@pytest.mark.parametrize("name,lib", libs())
def test_e2m1_table(name, lib):
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for code in range(16):
        want = mags[code] if code < 8 else -mags[code - 8]
        got = fn(lib, "e2m1")(code)
        assert got == want and math.copysign(1, got) == math.copysign(1, want)


@pytest.mark.parametrize("name,lib", libs())
def test_e4m3_all_codes(name, lib):
    dec = fn(lib, "e4m3_to_f32")
    assert dec(0x38) == 1.0 and dec(0x40) == 2.0 and dec(0x08) == 0.015625 and dec(0x30) == 0.5
    assert math.isnan(dec(0x7F)) and math.isnan(dec(0xFF))
    assert dec(0x80) == 0.0 and math.copysign(1, dec(0x80)) < 0
    for b in range(256):
        want = independent_fp8(b)
        got = dec(b)
        if math.isnan(want):
            assert math.isnan(got)
        else:
            assert got == want and (got != 0 or math.copysign(1, got) == math.copysign(1, want))


@pytest.mark.parametrize("name,lib", libs())
def test_e4m3_encoder_quirks(name, lib):
    enc = fn(lib, "f32_to_e4m3")
    assert enc(float("nan")) == 0x7F
    assert enc(1000.0) == 0x7E and enc(448.0) == 0x7E and enc(-448.0) == 0xFE
    assert enc(1.0) == 0x38 and enc(-0.0) == 0x80
    # subnormal band: [15 * 2^-10, 2^-6) rounds v * 2^9 to 8 and is capped at 7
    for v in (15 * 2.0 ** -10, 0.0155, 2.0 ** -6 - 2.0 ** -20):
        assert enc(v) == 0x07
    assert enc(2.0 ** -6) == 0x08
    # round-trip every finite code (canonical zero)
    dec = fn(lib, "e4m3_to_f32")
    for b in range(256):
        v = dec(b)
        if math.isnan(v):
            continue
        assert enc(v) == b


def _dequant(lib, packed, scales, gscale, rows, cols, out):
    if hasattr(lib, "or_e2m1"):
        return lib.or_nvfp4_dequantize(P(packed), P(scales), gscale, rows, cols, P(out))
    return lib.ref_nvfp4_dequantize(P(packed), packed.size, P(scales), scales.size, gscale, rows, cols, P(out),
                                    out.size)


@pytest.mark.parametrize("name,lib", libs())
def test_dequant_kats(name, lib):
    # low nibble first (tests/test_nvfp4_decode.cpp:57-63)
    packed = np.array([0x21, 0, 0, 0, 0, 0, 0, 0], np.uint8)
    scales = np.array([0x38], np.uint8)
    w = np.zeros(16, np.float32)
    assert _dequant(lib, packed, scales, 1.0, 1, 16, w) == 0
    assert w[0] == 0.5 and w[1] == 1.0 and np.all(w[2:] == 0)
    x = np.zeros(16, np.float64)
    x[0] = x[1] = 1.0
    assert float(w.astype(np.float64) @ x) == pytest.approx(1.5, abs=1e-5)
    assert _dequant(lib, packed, scales, 2.0, 1, 16, w) == 0  # weight_scale_2 multiplies
    assert float(w.astype(np.float64) @ x) == pytest.approx(3.0, abs=1e-5)
    packed32 = np.full(16, 0x22, np.uint8)
    scales2 = np.array([0x38, 0x40], np.uint8)
    wide = np.zeros(32, np.float32)
    assert _dequant(lib, packed32, scales2, 1.0, 1, 32, wide) == 0
    assert wide[0] == 1.0 and wide[16] == 2.0
    assert float(wide.astype(np.float64).sum()) == pytest.approx(48.0, abs=1e-5)


@pytest.mark.parametrize("name,lib", libs())
def test_dequant_view_grid(name, lib):
    # 4x64 view, scales cycling 0x08/0x30/0x38/0x40, global 2 (tests/test_nvfp4_view.cpp:44-59)
    rows, cols = 4, 64
    packed = ((np.arange(rows * cols // 2) * 37) & 0xFF).astype(np.uint8)
    codes = np.array([0x08, 0x30, 0x38, 0x40], np.uint8)
    scales = codes[np.arange(rows * cols // 16) % 4]
    out = np.zeros(rows * cols, np.float32)
    assert _dequant(lib, packed, scales, 2.0, rows, cols, out) == 0
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for r in range(rows):
        for c in range(cols):
            byte = int(packed[r * cols // 2 + c // 2])
            code = byte & 15 if c % 2 == 0 else byte >> 4
            fp4 = mags[code] if code < 8 else -mags[code - 8]
            want = np.float32(np.float32(fp4) * np.float32(independent_fp8(int(scales[r * cols // 16 + c // 16]))) * np.float32(2.0))
            assert out[r * cols + c] == want


@pytest.mark.parametrize("name,lib", libs())
def test_dequant_rejects_without_writing(name, lib):
    p16 = np.zeros(8, np.uint8)
    s16 = np.array([0x30], np.uint8)
    out = np.full(16, 123.0, np.float32)
    for c in (8, 17, 18):  # (0 columns is covered by the row check below)
        assert _dequant(lib, np.zeros(16, np.uint8), np.zeros(2, np.uint8), 1.0, 1, c, out) != 0
    assert _dequant(lib, p16, s16, 1.0, 0, 16, out) != 0
    for g in (0.0, -0.0, -1.0, math.inf, math.nan, 1.4e-45):
        assert _dequant(lib, p16, s16, g, 1, 16, out) != 0
    for bad in (0x7F, 0xFF, 0xB8):
        assert _dequant(lib, p16, np.array([bad], np.uint8), 1.0, 1, 16, out) != 0
    assert np.all(out == 123.0)
    assert _dequant(lib, p16, np.array([0], np.uint8), 1.0, 1, 16, out) == 0  # zero block scales are valid
    assert np.all(out == 0.0)


@pytest.mark.parametrize("name,lib", libs())
def test_routed_expert_shapes_sum(name, lib):
    # [N, K] routed-expert geometries with 0x22 codes, 0x30 scales, global 2:
    # every weight is 1, so y == K (tests/test_nvfp4_view.cpp:129-137)
    for n, k in ((2048, 4096), (4096, 2048)):
        packed = np.full(n * k // 2, 0x22, np.uint8)
        scales = np.full(n * k // 16, 0x30, np.uint8)
        w = np.zeros(n * k, np.float32)
        assert _dequant(lib, packed, scales, 2.0, n, k, w) == 0
        y = w.reshape(n, k).astype(np.float64).sum(axis=1)
        assert np.all(y == k)


@pytest.mark.parametrize("name,lib", libs())
def test_swiglu_and_router_kats(name, lib):
    gate = np.array([0.0, 100.0, -2.0], np.float32)
    up = np.array([1.0, 100.0, -20.0], np.float32)
    h = np.zeros(3, np.float32)
    fn(lib, "swiglu_clamp")(P(gate), P(up), 3, 10.0, P(h))
    assert h[0] == pytest.approx(0.0, abs=1e-5)
    assert h[1] == pytest.approx(99.995460213, abs=1e-4)
    assert h[2] == pytest.approx(2.384058440, abs=1e-5)
    logits = np.array([0.0, 10.0, 3.0, 10.0, 1.0], np.float32)
    bias = np.zeros(5, np.float32)
    idx = np.zeros(2, np.int32)
    w = np.zeros(2, np.float32)
    fn(lib, "router_select")(P(logits), P(bias), 5, 2, 2.5, 1, P(idx), P(w))
    assert list(idx) == [1, 3]  # the lower index wins the tie
    assert w[0] == pytest.approx(1.25, abs=1e-5) and w[1] == pytest.approx(1.25, abs=1e-5)


@pytest.mark.parametrize("name,lib", libs())
def test_mhc_combine_kat(name, lib):
    residual = np.array([0.5, 1.5], np.float32)
    branch = np.array([2.0], np.float32)
    post = np.array([1.0, 1.0], np.float32)
    comb = np.full(4, 0.5, np.float32)
    out = np.zeros(2, np.float32)
    fn(lib, "mhc_combine")(P(residual), P(branch), P(post), P(comb), 2, 1, P(out))
    assert out[0] == pytest.approx(3.0, abs=1e-5) and out[1] == pytest.approx(3.0, abs=1e-5)


@pytest.mark.parametrize("name,lib", libs())
def test_tiny_layer_kat(name, lib):
    width = 16
    packed = np.zeros(width * width // 2, np.uint8)
    packed[0] = 0x21
    scales = np.zeros(width * width // 16, np.uint8)
    scales[0] = 0x38
    weight = np.zeros(width * width, np.float32)
    assert _dequant(lib, packed, scales, 1.0, width, width, weight) == 0
    x = (0.25 * np.arange(1, width + 1)).astype(np.float32)
    nw = np.ones(width, np.float32)
    y = np.zeros(width, np.float32)
    normed = np.zeros(width, np.float32)
    fn(lib, "dense_residual_proj")(P(x), P(nw), P(weight), 1e-5, width, P(y))
    fn(lib, "rmsnorm")(P(x), P(nw), 1e-5, width, P(normed))
    expected0 = x[0] + weight[0] * normed[0] + weight[1] * normed[1]
    assert abs(y[0] - expected0) < 1e-5
    assert abs(weight[0] - 0.5) < 1e-5 and abs(weight[1] - 1.0) < 1e-5
    # width > 64 is a silent no-op (src/tiny_layer.cpp:17)
    big = np.full(65, 7.0, np.float32)
    fn(lib, "dense_residual_proj")(P(np.ones(65, np.float32)), P(np.ones(65, np.float32)),
                                   P(np.ones(65 * 65, np.float32)), 1e-5, 65, P(big))
    assert np.all(big == 7.0)


def test_quant_rejects_bad_scale():
    lib = orc.port()
    x = np.ones(16, np.float32)
    y = np.zeros(16, np.float32)
    for s in (0.0, -1.0, math.inf, math.nan):
        assert lib.or_quant_nvfp4_activation(P(x), 16, s, P(y), None, None) != 0
    assert lib.or_quant_nvfp4_activation(P(np.ones(17, np.float32)), 17, 1.0, P(np.zeros(17, np.float32)), None, None) != 0
