"""Synthetic input generator: its E4M3 / BF16 encoders agree with the
reference's rounding, and the configurations have the benchmark's shapes."""
import numpy as np

from helpers import oracle, workload

orc, wl = oracle(), workload()


def test_e4m3_encoder_matches_reference_on_normal_range():
    lib = orc.port()
    rng = np.random.Generator(np.random.PCG64(3))
    v = np.concatenate([np.clip(np.abs(rng.standard_normal(20000)), 2 ** -6, 448),
                        [2 ** -6, 448.0, 1.0, 1.0625, 1.1875, 240.0, 464.0 - 1e-3]]).astype(np.float32)
    v = np.minimum(v, np.float32(448))
    got = wl.e4m3_encode_normal(v)
    want = np.array([lib.or_f32_to_e4m3(float(a)) for a in v], np.uint8)
    assert np.array_equal(got, want)


def test_bf16_encoder_matches_reference():
    lib = orc.port()
    rng = np.random.Generator(np.random.PCG64(4))
    v = (rng.standard_normal(20000) * 10).astype(np.float32)
    got = wl.f32_to_bf16_bits(v)
    want = np.array([lib.or_f32_to_bf16(float(a)) for a in v], np.uint16)
    assert np.array_equal(got, want)


def test_config_shapes():
    lay, x = wl.config_layer("c0")
    assert x.shape == (16, 256) and lay.gate_packed.shape == (8, 128, 128) and lay.down_scales.shape == (8, 256, 8)
    assert lay.top_k == 2 and lay.scaling == 1.0
    assert float(lay.gate_ws2[0]) == np.float32(1) / np.float32(448)
    assert float(lay.gate_in[0]) == np.float32(1) / np.float32(6)


def test_zipf_bias_prefers_low_experts():
    lay, _ = wl.config_layer("c0")
    b = wl.zipf_bias(lay)
    assert b[0] > b[-1]


def test_c3_calibrated_lambda():
    """c3's calibrated log-prior weight is the grid point whose pick shares come
    closest to Zipf(1.1); at the literal lambda = 1 experts 0-3 take nearly every
    pick."""
    cfg = wl.CONFIGS["c3"]
    lay, x = wl.make_layer(cfg, 3), wl.make_tokens(cfg, 3)
    assert wl.calibrate_zipf_lambda(lay, x) == wl.C3_LAMBDA_CALIBRATED
    scores = wl._approx_choice(lay, x)

    def share_0_3(lam):
        top = np.argpartition(-(scores + wl.zipf_bias(lay, lam=lam)[None, :]), 3, axis=1)[:, :4]
        return np.isin(top, [0, 1, 2, 3]).mean()

    assert share_0_3(1.0) > 0.9
    assert 0.4 < share_0_3(wl.C3_LAMBDA_CALIBRATED) < 0.55
    lay1, _ = wl.config_layer("c3")
    assert np.array_equal(lay1.bias, wl.zipf_bias(lay, lam=1.0))
