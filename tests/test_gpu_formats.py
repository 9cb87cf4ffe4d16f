"""GPU format kernels against the oracle, bit for bit:
NVFP4 dequantisation (Nvfp4MatrixView::at), the activation quantiser
(quant_dequant_nvfp4_activation codes, scales and fake-quant values) and the
reference sigmoid (libm expf semantics) used by the router."""
import numpy as np
import pytest

from helpers import nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
orc, wl, m = oracle(), workload(), nfm()
P = orc.p


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_dequant_random_and_grid():
    rng = np.random.Generator(np.random.PCG64(20))
    for rows, cols, gs in ((4, 64, 2.0), (128, 512, 1 / 448), (37, 4096, 3.5)):
        packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
        scales = rng.integers(0, 0x7F, rows * cols // 16, dtype=np.uint8)  # every finite non-negative code
        want = np.zeros(rows * cols, np.float32)
        assert orc.port().or_nvfp4_dequantize(P(packed), P(scales), gs, rows, cols, P(want)) == 0
        out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        assert m.dequantize(dev(packed), dev(scales), gs, rows, cols, out) == 0
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_dequant_rejections():
    p16 = dev(np.zeros(8, np.uint8))
    out = torch.full((16,), 123.0, device="cuda")
    for bad in (0x7F, 0xFF, 0xB8):
        assert m.dequantize(p16, dev(np.array([bad], np.uint8)), 1.0, 1, 16, out) != 0
    for g in (0.0, -1.0, float("inf"), float("nan"), 1.4e-45):
        assert m.dequantize(p16, dev(np.array([0x30], np.uint8)), g, 1, 16, out) != 0
    assert m.dequantize(p16, dev(np.array([0x30], np.uint8)), 1.0, 1, 17, out) != 0
    assert torch.all(out == 123.0)


def test_routed_expert_shape_sums_to_k():
    n, k = 2048, 4096
    packed = dev(np.full(n * k // 2, 0x22, np.uint8))
    scales = dev(np.full(n * k // 16, 0x30, np.uint8))
    out = torch.empty(n * k, dtype=torch.float32, device="cuda")
    assert m.dequantize(packed, scales, 2.0, n, k, out) == 0
    assert torch.all(out.view(n, k).double().sum(dim=1) == k)


def quant_rows(rng):
    rows = [rng.standard_normal(512).astype(np.float32) * np.float32(s) for s in (1e-7, 1e-4, 1e-2, 0.3, 1, 7, 300)]
    special = rng.standard_normal(512).astype(np.float32)
    special[5] = np.nan
    special[40] = np.inf
    special[100] = -np.inf
    special[200:216] = 0.0
    special[216:232] = -0.0
    special[300:316] = np.float32(15 * 2.0 ** -10) * np.float32(6)  # E4M3 subnormal cap band
    rows.append(special)
    ties = np.tile(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, 6.0],
                            np.float32), 32)
    rows.append(ties)
    return np.stack(rows)


@pytest.mark.parametrize("input_scale", [1 / 6, 1.0, 0.01, 50.0])
def test_quantiser_bit_exact(input_scale):
    rng = np.random.Generator(np.random.PCG64(21))
    x = quant_rows(rng)
    fake, codes, scales = orc.quant_codes(orc.port(), x, np.float32(input_scale))
    xd = dev(x)
    c = torch.empty((x.shape[0], x.shape[1] // 2), dtype=torch.uint8, device="cuda")
    s = torch.empty((x.shape[0], x.shape[1] // 16), dtype=torch.uint8, device="cuda")
    f = torch.empty_like(xd)
    assert m.quantize(xd, x.shape[0], x.shape[1], float(np.float32(input_scale)), c, s, f) == 0
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy(), scales)
    assert np.array_equal(c.cpu().numpy(), codes)
    assert np.array_equal(f.cpu().numpy().view(np.uint32), fake.view(np.uint32))


def test_quantiser_rejects_bad_scale():
    x = dev(np.ones((1, 16), np.float32))
    c = torch.empty(8, dtype=torch.uint8, device="cuda")
    s = torch.empty(1, dtype=torch.uint8, device="cuda")
    for bad in (0.0, -1.0, float("inf"), float("nan")):
        assert m.quantize(x, 1, 16, bad, c, s) != 0
    assert m.quantize(x, 1, 17, 1.0, c, s) != 0


def _check_sigmoid(x: np.ndarray):
    want = orc.sigmoid_array(x)
    xd = dev(x)
    y = torch.empty_like(xd)
    assert m.sigmoid_ref(xd, x.size, y) == 0
    got = y.cpu().numpy()
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size == 0, f"{bad.size} sigmoid mismatches, first x={x[bad[:5]]}"


def test_sigmoid_random():
    rng = np.random.Generator(np.random.PCG64(22))
    _check_sigmoid(np.concatenate([rng.standard_normal(4_000_000).astype(np.float32) * np.float32(s) for s in (0.5, 2, 8)]
                                  + [rng.uniform(-120, 120, 1_000_000).astype(np.float32)]))


def test_sigmoid_full_binades():
    # every float of the binades that hold typical router logits, both signs
    parts = []
    for e in range(-3, 4):
        lo = np.float32(2.0 ** e).view(np.uint32)
        bits = np.arange(lo, lo + (1 << 23), dtype=np.uint32)
        parts.append(bits.view(np.float32))
        parts.append(-bits.view(np.float32))
    _check_sigmoid(np.concatenate(parts))


def test_hardware_conversions_match_reference_encoders():
    """The kernels use cvt.rn.satfinite e2m1x2 / e4m3x2 and cvt.rn.bf16(x2);
    over every 32-bit pattern they must agree with cast_to_e2m1 (after the
    +-6 clamp), f32_to_e4m3 on [2^-6, inf) (after the 448 clamp) and
    f32_to_bf16 on every non-NaN input."""
    e2m1, e4m3, bf16 = m.format_selfcheck()
    assert e2m1 == 0, f"{e2m1} E2M1 mismatches"
    assert e4m3 == 0, f"{e4m3} E4M3 mismatches"
    assert bf16 == 0, f"{bf16} BF16 rounding mismatches"
