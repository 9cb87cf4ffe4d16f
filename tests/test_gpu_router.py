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


# ---- the screened router of large batches --------------------------------------

def screened_forward(lay, x_bits):
    """A forward of a batch large enough for the screened router; returns the
    routes, the tensor-core logits it screened with and the candidate counts."""
    T = x_bits.shape[0]
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    y = torch.empty((T, lay.hidden), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, lay.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, lay.top_k), dtype=torch.float32, device="cuda")
    layer.forward(x, y, T, None, idx, w)
    layer.sync()
    approx = layer.debug_read("logits", np.float32, T * lay.experts).reshape(T, lay.experts)
    counts = layer.debug_read("screen_count", np.int32, T)
    out = idx.cpu().numpy(), w.cpu().numpy(), approx, counts
    layer.close()
    return out


def test_screened_router_prefill_bit_exact_with_bound_slack():
    """configs[2] through the forward (screened router): every route and weight
    bit-exact; the tensor cores' logit error, per ||x||_2 ||w_e||_2, stays far
    below the constant the screen's bound assumes for it; few chains run."""
    lay, x_bits = wl.config_layer("c2")
    idx, w, approx, counts = screened_forward(lay, x_bits)
    x = wl.bf16_bits_to_f32(x_bits)
    lg, want_idx, want_w = orc.route_tokens(lay, x)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    wn = np.sqrt((wl.bf16_bits_to_f32(lay.router_w).astype(np.float64) ** 2).sum(1))
    xn = np.sqrt((x.astype(np.float64) ** 2).sum(1))
    ratio = np.abs(approx.astype(np.float64) - lg) / (xn[:, None] * wn[None, :])
    H = lay.hidden
    assumed_tc = H * 2.0 ** -22  # the screen's allowance for the tensor-core accumulation
    assert ratio.max() < assumed_tc / 4, ratio.max()
    assert np.all(counts[counts >= 0] >= lay.top_k) and np.mean(counts < 0) < 0.01
    assert np.mean(counts[counts > 0]) < 16


def test_screened_router_exact_ties_and_special_tokens():
    """Duplicated router rows give exact ties at the top-k boundary (lowest
    index wins); NaN, infinite and huge token values take every chain.  Routes
    bit-exact against the oracle on a 1,536-token batch."""
    cfg = dict(wl.CONFIGS["c1"])
    lay = wl.make_layer(cfg, seed=21)
    for a, b in ((3, 40), (5, 6), (17, 60)):
        lay.router_w[b] = lay.router_w[a]
        lay.bias[b] = lay.bias[a]
    x_bits = wl.make_tokens(cfg, seed=21, tokens=1536).copy()
    x_bits[7, 100] = 0x7FC0                                                     # NaN
    x_bits[8, 5] = 0x7F80                                                       # +inf
    x_bits[9] = (x_bits[9].astype(np.uint32) + (40 << 7)).astype(np.uint16)     # x 2^40
    x_bits[10, 3] = 0x0001                                                      # BF16 subnormal
    idx, w, _, counts = screened_forward(lay, x_bits)
    _, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(idx, want_idx)
    ok = ~np.isnan(want_w).any(axis=1)
    assert np.array_equal(w[ok].view(np.uint32), want_w[ok].view(np.uint32))
    assert np.all(np.isnan(w[~ok]))
    assert all(counts[t] == -1 for t in (7, 8, 9, 10))
    # the tied pairs both reach the exact stage whenever one of them is near the boundary
    picks = set(map(tuple, np.sort(idx, axis=1)))
    assert any(3 in p for p in picks) and any(5 in p for p in picks)
