"""Router kernels (gemv_bf16 logits + router_select) against the oracle:
logits, indices and weights bit for bit, ties, group-limited routing."""
import numpy as np
import pytest

from helpers import nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
orc, wl, m = oracle(), workload(), nfm()


def run_router(lay, x_bits, n_group=1, topk_group=1):
    T = x_bits.shape[0]
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, n_group=n_group, topk_group=topk_group, max_tokens=T)
    layer.bind_layer(lay)
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    logits = torch.empty((T, lay.experts), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, lay.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, lay.top_k), dtype=torch.float32, device="cuda")
    layer.route(x, T, logits, idx, w)
    layer.sync()
    out = logits.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()
    layer.close()
    return out


@pytest.mark.parametrize("cfg", ["c0", "c1"])
def test_router_bit_exact(cfg):
    lay, x_bits = wl.config_layer(cfg)
    lg, idx, w = run_router(lay, x_bits)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(lg.view(np.uint32), want_lg.view(np.uint32))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))


def test_router_prefill_bit_exact_and_balanced():
    lay, x_bits = wl.config_layer("c2")
    lg, idx, w = run_router(lay, x_bits)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(lg.view(np.uint32), want_lg.view(np.uint32))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    counts = np.bincount(idx.ravel(), minlength=lay.experts)
    assert np.all(np.abs(counts - 512) <= 51), counts


def test_router_ties_keep_lower_index():
    lay, x_bits = wl.config_layer("c0")
    lay.router_w[5] = lay.router_w[2]   # identical rows -> identical logits
    lay.router_w[7] = lay.router_w[2]
    lay.bias[:] = 0.0
    lay.bias[2] = lay.bias[5] = lay.bias[7] = 5.0  # the tied experts win every token
    lg, idx, w = run_router(lay, x_bits)
    assert np.all(idx[:, 0] == 2) and np.all(idx[:, 1] == 5)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(idx, want_idx) and np.array_equal(w.view(np.uint32), want_w.view(np.uint32))


def test_router_group_limited():
    lay, x_bits = wl.config_layer("c1")
    lg, idx, w = run_router(lay, x_bits, n_group=8, topk_group=2)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits), n_group=8, topk_group=2)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    groups = idx // 8
    assert all(len(set(g)) <= 2 for g in groups)


@pytest.mark.parametrize("experts,top_k", [(96, 6), (160, 6)])
def test_router_wide_expert_counts(experts, top_k):
    """96 experts: the fused kernel with three warps of expert lanes; 160: the
    two-kernel path for more than 128 experts.  37 tokens: a ragged tail."""
    cfg = dict(hidden=256, experts=experts, top_k=top_k, inter=128, shared_inter=128, scaling=1.5, tokens=37)
    lay = wl.make_layer(cfg, seed=11)
    x_bits = wl.make_tokens(cfg, seed=11)
    lg, idx, w = run_router(lay, x_bits)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(lg.view(np.uint32), want_lg.view(np.uint32))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))


def test_router_rows_outside_the_exact_product_range():
    """Token values whose products with the weights leave fp32's exact range
    (huge, tiny, infinite) take the separately rounded multiply-add; the
    results still match the reference bit for bit."""
    lay, x_bits = wl.config_layer("c1")
    x_bits = x_bits.copy()
    x_bits[3] = (x_bits[3].astype(np.uint32) + (80 << 7)).astype(np.uint16)  # x 2^80
    x_bits[5, 10] = 0x0d00                                                      # 2^-101
    x_bits[9, 7] = 0x7f80                                                       # +inf
    x_bits[60, 2047] = 0x0001                                                   # BF16 subnormal
    lg, idx, w = run_router(lay, x_bits)
    want_lg, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(lg.view(np.uint32), want_lg.view(np.uint32))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
