"""The whole MoE layer on the GPU against the reference (golden file) and the
oracle: routes bit-exact, permutation exact, activation codes bit-exact,
expert and layer outputs within the stated tolerance (max-abs <= 2e-2,
cosine >= 0.9995), ragged and edge cases."""
from pathlib import Path

import numpy as np
import pytest

from golden.make_golden import residual_for
from helpers import MAX_ABS, MIN_COS, assert_close, nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
orc, wl, m = oracle(), workload(), nfm()
GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "c0_reference.npz")


def make_layer(lay, max_tokens, **kw):
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, bf16_experts=lay.bf16_experts, max_tokens=max_tokens, **kw)
    layer.bind_layer(lay)
    return layer


def gpu_forward(layer, x_bits, residual=None):
    T, H = x_bits.shape
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, layer.desc.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.desc.top_k), dtype=torch.float32, device="cuda")
    res = None if residual is None else torch.from_numpy(residual).cuda()
    layer.forward(x, y, T, res, idx, w)
    layer.sync()
    return y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def fetch(layer, which, dtype, count):
    return layer.debug_read(which, dtype, count)


@pytest.mark.parametrize("tag,bf16", [("nvfp4", False), ("bf16", True)])
def test_c0_against_reference_golden(tag, bf16):
    lay, x_bits = wl.config_layer("c0", bf16_experts=bf16)
    layer = make_layer(lay, 16)
    y, idx, w = gpu_forward(layer, x_bits)
    assert np.array_equal(idx, GOLDEN[f"{tag}_idx"])
    assert np.array_equal(w.view(np.uint32), GOLDEN[f"{tag}_w"].view(np.uint32))
    assert_close(y, GOLDEN[f"{tag}_y"], what=f"c0 {tag} y")
    res = residual_for(x_bits)
    yr, _, _ = gpu_forward(layer, x_bits, res)
    assert_close(yr, GOLDEN[f"{tag}_y_residual"], what=f"c0 {tag} y+residual")
    layer.close()


def test_c1_against_oracle_and_stages():
    lay, x_bits = wl.config_layer("c1")
    T, H, K, E = x_bits.shape[0], lay.hidden, lay.top_k, lay.experts
    x = wl.bf16_bits_to_f32(x_bits)
    layer = make_layer(lay, T)
    y, idx, w = gpu_forward(layer, x_bits)
    want_y, want_idx, want_w, routed, shared = orc.moe_layer(orc.port(), lay, x, taps=True)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    assert_close(y, want_y, what="c1 y")
    # permutation: expert-major, token order inside a segment, 128-aligned segments
    counts = fetch(layer, "counts", np.int32, E)
    seg = fetch(layer, "seg_offset", np.int32, E + 1)
    pair_row = fetch(layer, "pair_row", np.int32, T * K).reshape(T, K)
    rows_used = int(fetch(layer, "rows", np.int32, 1)[0])
    row_token = fetch(layer, "row_token", np.int32, rows_used)
    assert np.array_equal(counts, np.bincount(idx.ravel(), minlength=E))
    padded = (counts + 127) // 128 * 128
    assert np.array_equal(seg, np.concatenate([[0], np.cumsum(padded)]).astype(np.int32))
    assert rows_used == seg[-1]
    for e in range(E):
        toks = np.nonzero((idx == e).any(axis=1))[0]
        rows = seg[e] + np.arange(toks.size)
        assert np.array_equal(row_token[rows], toks)
        assert np.all(row_token[seg[e] + toks.size: seg[e + 1]] == -1)
        for t, r in zip(toks, rows):
            p = int(np.nonzero(idx[t] == e)[0][0])
            assert pair_row[t, p] == r
    # dispatch codes: bit-exact against the oracle quantiser of each token
    codes = fetch(layer, "act_codes", np.uint8, rows_used * H // 2).reshape(rows_used, H // 2)
    sf_atoms = fetch(layer, "act_sf", np.uint8, rows_used * H // 16)
    sf = m.sf_from_atoms(sf_atoms, rows_used, H // 16)
    _, want_codes, want_sf = orc.quant_codes(orc.port(), x, float(lay.gate_in[0]))
    live = row_token >= 0
    assert np.array_equal(codes[live], want_codes[row_token[live]])
    assert np.array_equal(sf[live], want_sf[row_token[live]])
    # per-expert down outputs (BF16) against the oracle's linear_nvfp4 chain
    down = fetch(layer, "down", np.uint16, rows_used * H).reshape(rows_used, H)
    errs = []
    for t in range(0, T, 7):
        for p in range(K):
            _, want_d = orc.expert_forward(lay, int(idx[t, p]), x[t])
            got_d = wl.bf16_bits_to_f32(down[pair_row[t, p]])
            errs.append(np.max(np.abs(got_d - want_d)))
            assert_close(got_d, want_d, max_abs=MAX_ABS, min_cos=0.999, what=f"down t{t} p{p}")
    # shared expert output
    sh = fetch(layer, "shared", np.float32, T * H).reshape(T, H)
    assert_close(sh, shared, what="shared expert")
    layer.close()


def test_forward_host_matches_device_and_is_deterministic():
    lay, x_bits = wl.config_layer("c1")
    layer = make_layer(lay, 64)
    y1, i1, w1 = gpu_forward(layer, x_bits)
    y2, i2, w2 = gpu_forward(layer, x_bits)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    res = residual_for(x_bits)
    yh, ih, wh = layer.forward_host(wl.bf16_bits_to_f32(x_bits), res, with_routes=True)
    yd, _, _ = gpu_forward(layer, x_bits, res)
    assert np.array_equal(ih, i1) and np.array_equal(wh.view(np.uint32), w1.view(np.uint32))
    assert np.array_equal(yh.view(np.uint32), yd.view(np.uint32))
    # caller-owned (page-locked) output arrays, reused across calls
    outs = tuple(torch.from_numpy(np.empty_like(a)).pin_memory().numpy() for a in (yh, ih, wh))
    for _ in range(2):
        yo, io, wo = layer.forward_host(wl.bf16_bits_to_f32(x_bits), res, out=outs)
        assert yo is outs[0] and np.array_equal(yo.view(np.uint32), yh.view(np.uint32))
        assert np.array_equal(io, ih) and np.array_equal(wo.view(np.uint32), wh.view(np.uint32))
    # graph mode with every host buffer page-locked: copies and layer replay as one graph
    layer.set_graph_mode(True)
    xp = torch.from_numpy(wl.bf16_bits_to_f32(x_bits)).pin_memory().numpy()
    rp = torch.from_numpy(res).pin_memory().numpy()
    for _ in range(3):
        for a in outs:
            a.fill(0)
        yo, io, wo = layer.forward_host(xp, rp, out=outs)
        assert np.array_equal(yo.view(np.uint32), yh.view(np.uint32))
        assert np.array_equal(io, ih) and np.array_equal(wo.view(np.uint32), wh.view(np.uint32))
    layer.close()


def test_one_token_and_empty_and_capacity():
    lay, x_bits = wl.config_layer("c0")
    layer = make_layer(lay, 16)
    y, idx, w = gpu_forward(layer, x_bits[:1])
    want_y, want_idx, want_w = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits[:1]))
    assert np.array_equal(idx, want_idx)
    assert_close(y, want_y, what="T=1")
    x = torch.zeros((1, lay.hidden), dtype=torch.int16, device="cuda")
    yz = torch.empty((1, lay.hidden), dtype=torch.float32, device="cuda")
    layer.forward(x, yz, 0)  # zero tokens is a no-op
    layer.forward(None, None, 0)  # ... that reads and writes nothing, so it takes NULL buffers
    layer.route(None, 0)
    with pytest.raises(m.NfError, match="null input"):
        layer.forward(None, yz, 1)
    with pytest.raises(m.NfError, match="null output"):
        layer.forward(x, None, 1)
    with pytest.raises(RuntimeError, match="max_tokens"):
        layer.forward(x, yz, 17)
    layer.close()


def test_skewed_routing_many_tiles_per_expert():
    """All tokens on the same k experts (several 128-row tiles each), the
    other experts empty."""
    cfg = dict(wl.CONFIGS["c1"])
    lay = wl.make_layer(cfg, 5)
    lay.bias[:] = -10.0
    lay.bias[[3, 17, 40, 63]] = 10.0
    x_bits = wl.make_tokens(cfg, 5, tokens=300)
    layer = make_layer(lay, 300)
    y, idx, w = gpu_forward(layer, x_bits)
    assert set(np.unique(idx)) == {3, 17, 40, 63}
    sel = np.arange(0, 300, 13)
    want_y, want_idx, _ = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits[sel]))
    assert np.array_equal(idx[sel], want_idx)
    assert_close(y[sel], want_y, what="skewed")
    layer.close()


def test_ragged_expert_sizes():
    cfg = dict(wl.CONFIGS["c0"])
    lay = wl.make_layer(cfg, 9)
    rng = np.random.Generator(np.random.PCG64(9))
    lay.bias = rng.uniform(-2, 2, lay.experts).astype(np.float32)
    x_bits = wl.make_tokens(cfg, 9, tokens=333)
    layer = make_layer(lay, 333)
    y, idx, w = gpu_forward(layer, x_bits)
    want_y, want_idx, want_w = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    assert_close(y, want_y, what="ragged")
    layer.close()


def test_graph_mode_replays_bit_identical():
    lay, x_bits = wl.config_layer("c1")
    T, H, K = x_bits.shape[0], lay.hidden, lay.top_k
    layer = make_layer(lay, T)
    direct, _, _ = gpu_forward(layer, x_bits)
    layer.set_graph_mode(True)
    s = torch.cuda.Stream()
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    outs = []
    with torch.cuda.stream(s):
        for _ in range(3):  # capture, then two replays
            y.zero_()
            layer.forward(x, y, T, None, idx, w, stream=s.cuda_stream)
            layer.sync(s.cuda_stream)
            outs.append(y.cpu().numpy().copy())
    for o in outs:
        assert np.array_equal(o.view(np.uint32), direct.view(np.uint32))
    yh = layer.forward_host(wl.bf16_bits_to_f32(x_bits))  # host path through its own captured graph
    assert np.array_equal(yh.view(np.uint32), direct.view(np.uint32))
    layer.close()


def test_nan_token_routes_like_reference():
    """A NaN activation makes every logit NaN: the reference then keeps the
    first unused expert at each pick (its strict '>' scan never moves)."""
    lay, x_bits = wl.config_layer("c0")
    x_bits = x_bits.copy()
    x_bits[3, 17] = 0x7FC0  # BF16 NaN
    layer = make_layer(lay, 16)
    y, idx, w = gpu_forward(layer, x_bits)
    _, want_idx, want_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    assert np.array_equal(idx, want_idx)
    assert list(idx[3]) == list(range(lay.top_k))
    assert np.all(np.isnan(w[3])) and np.all(np.isnan(want_w[3]))
    ok = np.ones(16, bool)
    ok[3] = False
    assert np.array_equal(w[ok].view(np.uint32), want_w[ok].view(np.uint32))
    layer.close()


def test_misaligned_buffers_are_rejected_before_any_launch():
    lay, x_bits = wl.config_layer("c0")
    T = x_bits.shape[0]
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    xbuf = torch.zeros(T * lay.hidden + 8, dtype=torch.int16, device="cuda")
    y = torch.zeros((T, lay.hidden), dtype=torch.float32, device="cuda")
    with pytest.raises(m.NfError, match="16-byte aligned"):
        layer.forward(xbuf.data_ptr() + 2, y, T)   # x off by one BF16 element
    ybuf = torch.zeros(T * lay.hidden + 4, dtype=torch.float32, device="cuda")
    with pytest.raises(m.NfError, match="16-byte aligned"):
        layer.forward(xbuf, ybuf.data_ptr() + 4, T)
    layer.sync()
    layer.close()


def test_large_batch_shared_expert_paired_tiles():
    """From 2,048 tokens the shared expert's BF16 GEMMs use 256-row tiles (two
    accumulators per B stage): its output and the layer's against the oracle,
    on a ragged batch whose last tile holds 52 rows."""
    cfg = dict(wl.CONFIGS["c0"])
    lay = wl.make_layer(cfg, seed=31)
    x_bits = wl.make_tokens(cfg, seed=31, tokens=2100)
    T, H = x_bits.shape
    layer = make_layer(lay, T)
    y, idx, w = gpu_forward(layer, x_bits)
    want_y, want_idx, _, _, shared = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits), taps=True)
    assert np.array_equal(idx, want_idx)
    sh = fetch(layer, "shared", np.float32, T * H).reshape(T, H)
    assert_close(sh, shared, what="shared expert, 256-row tiles")
    assert_close(y, want_y, what="layer, T = 2100")
    layer.close()


def test_bf16_experts_c1_against_oracle():
    """The BF16 routed experts (the layer-45 form, whose oracle is mlp_bf16 per
    expert) at the decode batch's full shapes: routes bit-exact, layer output
    and residual form within the tolerance."""
    lay, x_bits = wl.config_layer("c1", bf16_experts=True)
    x = wl.bf16_bits_to_f32(x_bits)
    layer = make_layer(lay, x_bits.shape[0])
    y, idx, w = gpu_forward(layer, x_bits)
    want_y, want_idx, want_w = orc.moe_layer(orc.port(), lay, x)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    assert_close(y, want_y, what="c1 BF16 experts")
    res = residual_for(x_bits)
    yr, _, _ = gpu_forward(layer, x_bits, res)
    want_r, _, _ = orc.moe_layer(orc.port(), lay, x, res)
    assert_close(yr, want_r, what="c1 BF16 experts + residual")
    layer.close()


def test_group_limited_routing_through_the_layer():
    """Group-limited top-k (8 groups of 8 experts, 4 kept) through the whole
    layer: routes bit-exact against the oracle's group-limited selection and
    the output within the tolerance."""
    lay, x_bits = wl.config_layer("c1")
    x = wl.bf16_bits_to_f32(x_bits)
    layer = make_layer(lay, x_bits.shape[0], n_group=8, topk_group=4)
    y, idx, w = gpu_forward(layer, x_bits)
    want_y, want_idx, want_w = orc.moe_layer(orc.port(), lay, x, n_group=8, topk_group=4)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    # every pick lies in one of the token's 4 kept groups
    assert np.all(np.array([np.unique(r // 8).size for r in idx]) <= 4)
    assert_close(y, want_y, what="c1 group-limited")
    layer.close()


def test_c2_prefill_layer_at_its_configuration():
    """configs[2] exactly: 8192 tokens, H2048, the tuned bias, through the
    large-batch permutation and dispatch path.  All 8192 routes and weights
    bit-exact against the oracle's router; the E2M1 codes and E4M3 scales of
    every live dispatched row bit-exact against the oracle's quantiser of its
    token; the permutation exact; the layer output within the tolerance on a
    deterministic subset of 135 tokens (tokens are independent, so a subset
    is a full check of those tokens), with their down rows."""
    lay, x_bits = wl.config_layer("c2")
    T, H, K, E = x_bits.shape[0], lay.hidden, lay.top_k, lay.experts
    x = wl.bf16_bits_to_f32(x_bits)
    layer = make_layer(lay, T)
    y, idx, w = gpu_forward(layer, x_bits)
    _, want_idx, want_w = orc.route_tokens(lay, x)
    assert np.array_equal(idx, want_idx)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    counts = np.bincount(idx.ravel(), minlength=E)
    assert np.all(np.abs(counts - 512) <= 51), counts
    # permutation: expert-major, token order inside a segment, 128-aligned segments
    seg = fetch(layer, "seg_offset", np.int32, E + 1)
    padded = (counts + 127) // 128 * 128
    assert np.array_equal(seg, np.concatenate([[0], np.cumsum(padded)]).astype(np.int32))
    rows_used = int(fetch(layer, "rows", np.int32, 1)[0])
    assert rows_used == seg[-1]
    row_token = fetch(layer, "row_token", np.int32, rows_used)
    pair_row = fetch(layer, "pair_row", np.int32, T * K).reshape(T, K)
    for e in range(E):
        toks = np.nonzero((idx == e).any(axis=1))[0]
        assert np.array_equal(row_token[seg[e]:seg[e] + toks.size], toks)
        assert np.all(row_token[seg[e] + toks.size:seg[e + 1]] == -1)
    p_of = np.argmax(idx[:, :, None] == np.arange(E)[None, None, :], axis=1)  # [T, E]: pick of expert e
    tt, kk = np.meshgrid(np.arange(T), np.arange(K), indexing="ij")
    assert np.array_equal(row_token[pair_row], tt)
    assert np.all(p_of[tt, idx] == kk)
    # dispatched activation codes and scales of every live row
    codes = fetch(layer, "act_codes", np.uint8, rows_used * H // 2).reshape(rows_used, H // 2)
    sf = m.sf_from_atoms(fetch(layer, "act_sf", np.uint8, rows_used * H // 16), rows_used, H // 16)
    _, want_codes, want_sf = orc.quant_codes(orc.port(), x, float(lay.gate_in[0]))
    live = row_token >= 0
    assert int(live.sum()) == T * K
    assert np.array_equal(codes[live], want_codes[row_token[live]])
    assert np.array_equal(sf[live], want_sf[row_token[live]])
    # layer output and down rows on a deterministic subset
    sel = np.arange(0, T, 61)
    assert sel.size >= 128
    want_y, sel_idx, _ = orc.moe_layer(orc.port(), lay, x[sel])
    assert np.array_equal(sel_idx, idx[sel])
    assert_close(y[sel], want_y, what="c2 y (subset)")
    down = fetch(layer, "down", np.uint16, rows_used * H).reshape(rows_used, H)
    for t in sel[::9]:
        for p in range(K):
            _, want_d = orc.expert_forward(lay, int(idx[t, p]), x[t])
            assert_close(wl.bf16_bits_to_f32(down[pair_row[t, p]]), want_d, max_abs=MAX_ABS, min_cos=0.999,
                         what=f"c2 down t{t} p{p}")
    layer.close()
