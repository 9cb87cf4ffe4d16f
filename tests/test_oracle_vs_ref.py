"""The C restatement (oracle/nf_oracle.c) must equal the reference's own
sources (oracle/_ref, compiled from the reference tree) bit for bit on the
same inputs.  Skipped where the reference library was not built."""
import ctypes

import numpy as np
import pytest

from helpers import oracle, workload

orc = oracle()
wl = workload()
P = orc.p
REF = orc.ref()
PORT = orc.port()
pytestmark = pytest.mark.skipif(REF is None, reason="reference sources not built (oracle/_ref)")


def interesting_floats(rng, n=200_000):
    """Random bit patterns plus values around format boundaries."""
    bits = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    extra = np.array([0.0, -0.0, 448.0, 449.0, 464.0, 480.0, 2.0 ** -6, 2.0 ** -7, 15 * 2.0 ** -10, 2.0 ** -9,
                      2.0 ** -10, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, np.inf, -np.inf, np.nan], np.float32)
    normal = rng.standard_normal(n).astype(np.float32) * np.float32(4.0)
    return np.concatenate([f, extra, -extra, normal])


def test_scalar_formats_bit_exact():
    rng = np.random.Generator(np.random.PCG64(7))
    xs = interesting_floats(rng, 50_000)
    for v in xs[:120_000]:
        v = float(v)
        assert PORT.or_f32_to_e4m3(v) == REF.ref_f32_to_e4m3(v)
        assert PORT.or_f32_to_bf16(v) == REF.ref_f32_to_bf16(v)
        a, b = PORT.or_cast_to_e2m1(v), REF.ref_cast_to_e2m1(v)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_sigmoid_bit_exact():
    rng = np.random.Generator(np.random.PCG64(8))
    xs = np.concatenate([rng.standard_normal(100_000).astype(np.float32) * np.float32(3),
                         rng.uniform(-100, 100, 20_000).astype(np.float32)])
    for v in xs:
        a, b = PORT.or_sigmoid(float(v)), REF.ref_sigmoid(float(v))
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_quant_dequant_bit_exact():
    rng = np.random.Generator(np.random.PCG64(9))
    rows = [rng.standard_normal(256).astype(np.float32) * np.float32(s) for s in (1e-6, 1e-3, 0.1, 1, 10, 1e4)]
    special = np.zeros(256, np.float32)
    special[3] = np.nan
    special[20] = np.inf
    special[40] = -np.inf
    special[60:76] = 2.0 ** -12
    rows += [special, np.zeros(256, np.float32)]
    for x in rows:
        for s in (1 / 6, 1.0, 1e-3, 37.0):
            ya = np.zeros(256, np.float32)
            yb = np.zeros(256, np.float32)
            assert PORT.or_quant_nvfp4_activation(P(x), 256, s, P(ya), None, None) == 0
            assert REF.ref_quant_dequant(P(x), 256, s, P(yb)) == 0
            assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


def test_gemvs_bit_exact():
    rng = np.random.Generator(np.random.PCG64(10))
    rows, cols = 96, 512
    packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    scales = wl.e4m3_encode_normal(np.clip(np.abs(rng.standard_normal(rows * cols // 16)), 2 ** -6, 448).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    ya, yb = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    PORT.or_gemv_nvfp4_rows(P(packed), P(scales), 1 / 448, 1 / 6, P(x), rows, cols, 0, rows, P(ya))
    REF.ref_gemv_nvfp4_rows(P(packed), P(scales), 1 / 448, 1 / 6, P(x), rows, cols, 0, rows, P(yb))
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
    w = wl.f32_to_bf16_bits(rng.standard_normal(rows * cols).astype(np.float32))
    PORT.or_gemv_bf16(P(w), P(x), rows, cols, 0, rows, P(ya))
    REF.ref_gemv_bf16(P(w), P(x), rows, cols, 0, rows, P(yb))
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


def test_router_select_bit_exact():
    rng = np.random.Generator(np.random.PCG64(11))
    for trial in range(3000):
        E = int(rng.choice([5, 8, 64, 288]))
        k = int(rng.integers(1, min(E, 8) + 1))
        logits = rng.standard_normal(E).astype(np.float32)
        if trial % 5 == 0:  # plant ties
            logits[rng.integers(0, E, 3)] = logits[0]
        bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
        ia, ib = np.zeros(k, np.int32), np.zeros(k, np.int32)
        wa, wb = np.zeros(k, np.float32), np.zeros(k, np.float32)
        PORT.or_router_select(P(logits), P(bias), E, k, 2.5, 1, P(ia), P(wa))
        REF.ref_router_select(P(logits), P(bias), E, k, 2.5, 1, P(ib), P(wb))
        assert np.array_equal(ia, ib) and np.array_equal(wa.view(np.uint32), wb.view(np.uint32))
        # group-limited with one group is the plain router
        PORT.or_router_select_grouped(P(logits), P(bias), E, k, 2.5, 1, 1, 1, P(ia), P(wa))
        assert np.array_equal(ia, ib) and np.array_equal(wa.view(np.uint32), wb.view(np.uint32))


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Equal bit for bit, except that a NaN only has to meet a NaN: its payload
    follows the order of the operands that made it."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return bool(np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)))


def test_router_select_special_logits():
    """Non-finite and huge logits, with and without renormalisation: the
    reference's selection takes the first unused expert as its start and
    replaces it only on a strict ">", so a NaN choice at the lowest unused
    index is kept (no comparison against it succeeds) and ties keep the lower
    index."""
    rng = np.random.Generator(np.random.PCG64(15))
    specials = np.array([np.nan, np.inf, -np.inf, 3e38, -3e38, 1e-40, -0.0, 88.0, -88.0, 104.0], np.float32)
    for trial in range(2000):
        E = int(rng.choice([8, 16, 64]))
        k = int(rng.integers(1, min(E, 8) + 1))
        logits = rng.standard_normal(E).astype(np.float32)
        n_sp = int(rng.integers(1, 4))
        logits[rng.integers(0, E, n_sp)] = rng.choice(specials, n_sp)
        if trial % 7 == 0:
            logits[0] = np.nan  # the first expert scanned
        bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
        if trial % 11 == 0:
            bias[rng.integers(0, E)] = np.float32(np.inf)
        normalize, scaling = int(trial % 3 != 0), float(rng.choice([1.0, 2.5]))
        ia, ib = np.zeros(k, np.int32), np.zeros(k, np.int32)
        wa, wb = np.zeros(k, np.float32), np.zeros(k, np.float32)
        PORT.or_router_select(P(logits), P(bias), E, k, scaling, normalize, P(ia), P(wa))
        REF.ref_router_select(P(logits), P(bias), E, k, scaling, normalize, P(ib), P(wb))
        assert np.array_equal(ia, ib), (trial, logits, ia, ib)
        assert same_bits(wa, wb), (trial, wa, wb)


def test_gemvs_out_of_range_values_bit_exact():
    """Both GEMVs on values whose products leave fp32's exact range (huge,
    tiny, subnormal), overflow to infinity, or carry NaN and infinity: the
    restatement still follows the reference's rounding step by step."""
    rng = np.random.Generator(np.random.PCG64(16))
    rows, cols = 64, 256
    x = rng.standard_normal(cols).astype(np.float32)
    x[3], x[17], x[40], x[41], x[99] = 2.0 ** 100, 2.0 ** -120, 1e-42, -3e38, np.float32(2.0 ** 60)
    for special in (None, np.inf, np.nan):
        xs = x.copy()
        if special is not None:
            xs[200] = special
        w = wl.f32_to_bf16_bits(rng.standard_normal(rows * cols).astype(np.float32))
        w[::97] = 0x7E80  # ~8.5e37
        w[5::89] = 0x0001  # BF16 subnormal
        ya, yb = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
        PORT.or_gemv_bf16(P(w), P(xs), rows, cols, 0, rows, P(ya))
        REF.ref_gemv_bf16(P(w), P(xs), rows, cols, 0, rows, P(yb))
        assert same_bits(ya, yb)
        packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
        scales = wl.e4m3_encode_normal(np.clip(np.abs(rng.standard_normal(rows * cols // 16)), 2 ** -6, 448)
                                       .astype(np.float32))
        for in_scale in (1 / 6, 1e-30, 1e30):
            PORT.or_gemv_nvfp4_rows(P(packed), P(scales), 1 / 448, in_scale, P(xs), rows, cols, 0, rows, P(ya))
            REF.ref_gemv_nvfp4_rows(P(packed), P(scales), 1 / 448, in_scale, P(xs), rows, cols, 0, rows, P(yb))
            assert same_bits(ya, yb)


def test_swiglu_bit_exact():
    rng = np.random.Generator(np.random.PCG64(12))
    g = (rng.standard_normal(4096) * 8).astype(np.float32)
    u = (rng.standard_normal(4096) * 8).astype(np.float32)
    g[:4] = [np.nan, np.inf, -np.inf, 10.0]
    for name in ("swiglu_clamp", "swiglu_clamp_bf16"):
        ha, hb = np.zeros(4096, np.float32), np.zeros(4096, np.float32)
        getattr(PORT, "or_" + name)(P(g), P(u), 4096, 10.0, P(ha))
        getattr(REF, "ref_" + name)(P(g), P(u), 4096, 10.0, P(hb))
        assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32))


@pytest.mark.parametrize("bf16_experts", [False, True])
def test_moe_layer_c0_bit_exact(bf16_experts):
    lay, x_bits = wl.config_layer("c0", bf16_experts=bf16_experts)
    x = wl.bf16_bits_to_f32(x_bits)
    res = np.random.Generator(np.random.PCG64(13)).standard_normal(x.shape).astype(np.float32)
    for residual in (None, res):
        ya, ia, wa = orc.moe_layer(PORT, lay, x, residual)
        yb, ib, wb = orc.moe_layer(REF, lay, x, residual)
        assert np.array_equal(ia, ib)
        assert np.array_equal(wa.view(np.uint32), wb.view(np.uint32))
        assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


def test_moe_layer_c1_subset_bit_exact():
    lay, x_bits = wl.config_layer("c1")
    x = wl.bf16_bits_to_f32(x_bits[:3])
    ya, ia, wa = orc.moe_layer(PORT, lay, x)
    yb, ib, wb = orc.moe_layer(REF, lay, x)
    assert np.array_equal(ia, ib) and np.array_equal(wa.view(np.uint32), wb.view(np.uint32))
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


@pytest.mark.parametrize("hidden,inter,tokens", [(256, 512, 9), (2048, 10240, 2)])
def test_dense_mlp_bit_exact(hidden, inter, tokens):
    """dense_mlp (src/text_forward.cpp:909-915): the restatement against the
    reference's own primitives, with and without the residual; the second
    case has the dense layers' shapes of the benchmark's decoder stack."""
    lay = wl.make_dense_layer(hidden, inter, seed=40 + tokens)
    x = wl.bf16_bits_to_f32(wl.make_tokens(dict(hidden=hidden, tokens=tokens), 40 + tokens))
    res = np.random.Generator(np.random.PCG64(14)).standard_normal(x.shape).astype(np.float32)
    for residual in (None, res):
        ya = orc.dense_mlp(PORT, lay, x, residual)
        yb = orc.dense_mlp(REF, lay, x, residual)
        assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
