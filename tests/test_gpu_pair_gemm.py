"""The alternative forms of the grouped NVFP4 expert GEMMs at prefill sizes
(nf_moe_set_expert_gemm): CTA pairs (tcgen05 cta_group::2, 256-row tiles,
activation rows resident; nf_gemm2.cu) and 512-K stages of the one-SM kernel,
against the default one-SM kernel on the same inputs (the intermediate h codes
and scales, the down rows), and the layer against the oracle (routes bit-exact, output within
max-abs 2e-2 / cosine 0.9995) on ragged segments: empty experts, experts
with fewer than 128 rows, odd numbers of 128-row blocks (a pair tile whose
second CTA holds no rows of the expert) and several pair tiles per expert."""
import numpy as np
import pytest

from helpers import assert_close, nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
orc, wl, m = oracle(), workload(), nfm()


def make_layer(lay, max_tokens):
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=max_tokens)
    layer.bind_layer(lay)
    return layer


def forward(layer, x_bits):
    T, H = x_bits.shape
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, layer.desc.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.desc.top_k), dtype=torch.float32, device="cuda")
    layer.forward(x, y, T, None, idx, w)
    layer.sync()
    return y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def intermediates(layer, T, K, H, I):
    rows = int(layer.debug_read("rows", np.int32, 1)[0])
    row_token = layer.debug_read("row_token", np.int32, rows)
    live = row_token >= 0
    h = layer.debug_read("h_codes", np.uint8, rows * I // 2).reshape(rows, I // 2)[live]
    hs = m.sf_from_atoms(layer.debug_read("h_sf", np.uint8, rows * I // 16), rows, I // 16)[live]
    down = layer.debug_read("down", np.uint16, rows * H).reshape(rows, H)[live]
    return h, hs, down


def both_paths(lay, x_bits):
    T, H, K, I = x_bits.shape[0], lay.hidden, lay.top_k, lay.inter
    layer = make_layer(lay, T)
    layer.set_expert_gemm("pair")
    y2, idx2, w2 = forward(layer, x_bits)
    pair = intermediates(layer, T, K, H, I)
    layer.set_expert_gemm("wide")
    yw, idxw, ww = forward(layer, x_bits)
    wide = intermediates(layer, T, K, H, I)
    layer.set_expert_gemm("one_sm")
    y1, idx1, w1 = forward(layer, x_bits)
    one = intermediates(layer, T, K, H, I)
    layer.close()
    for i, wt in ((idx2, w2), (idxw, ww)):
        assert np.array_equal(idx1, i)
        assert np.array_equal(w1.view(np.uint32), wt.view(np.uint32))
    compare_paths(wide, one, "512-K stages")
    return (y2, idx2, w2, pair), (y1, one)


def compare_paths(pair, one, what):
    """The two kernels reduce each output's K in the same stage order; the
    h codes, their scales and the down rows agree bit for bit where the MMAs'
    fp32 results do, and the down rows within the layer tolerance in any
    case."""
    h2, hs2, d2 = pair
    h1, hs1, d1 = one
    mism = float(np.mean(h1 != h2))
    assert mism < 1e-3, f"{what}: {mism:.2e} of the h code bytes differ"
    assert float(np.mean(hs1 != hs2)) < 1e-3
    f = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
    assert_close(f(d2), f(d1), what=f"{what}: down rows, pair vs one-SM")


def test_pair_gemm_c2_against_one_sm_and_oracle():
    """configs[2] (8192 tokens, 512 +- 10% rows per expert: 4 or 5 blocks of
    128, so 2 or 3 pair tiles per expert, the last one often half empty)."""
    lay, x_bits = wl.config_layer("c2")
    (y2, idx, w, pair), (y1, one) = both_paths(lay, x_bits)
    compare_paths(pair, one, "c2")
    sel = np.arange(0, x_bits.shape[0], 61)
    want_y, want_idx, _ = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits[sel]))
    assert np.array_equal(idx[sel], want_idx)
    assert_close(y2[sel], want_y, what="c2 layer, pair GEMMs")
    assert_close(y1[sel], want_y, what="c2 layer, one-SM GEMMs")


def test_pair_gemm_ragged_segments():
    """H 512, I 256, 16 experts, top-2, 2300 tokens with a wide bias spread:
    segment sizes from 0 to well over 512 rows."""
    cfg = dict(hidden=512, experts=16, top_k=2, inter=256, shared_inter=256, tokens=2300, scaling=1.0)
    lay = wl.make_layer(cfg, 41)
    rng = np.random.Generator(np.random.PCG64(41))
    lay.bias = rng.uniform(-0.6, 0.6, lay.experts).astype(np.float32)
    lay.bias[5] = -10.0  # no rows
    lay.bias[9] = -0.9   # few rows
    x_bits = wl.make_tokens(cfg, 41, tokens=2300)
    (y2, idx, w, pair), (y1, one) = both_paths(lay, x_bits)
    counts = np.bincount(idx.ravel(), minlength=lay.experts)
    assert counts[5] == 0
    blocks = (counts + 127) // 128
    assert np.any(blocks % 2 == 1) and np.any(blocks >= 4), counts
    compare_paths(pair, one, "ragged")
    want_y, want_idx, want_w = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    assert_close(y2, want_y, what="ragged layer, pair GEMMs")
