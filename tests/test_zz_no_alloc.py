"""nf_router_topk_noalloc (router top-k with no device allocation, scratch in
a static device array) against the handle's nf_moe_route and against the CPU
oracle's router (gemv_bf16 + router_select restated, pinned to the
reference) on the same inputs: indices equal and weights equal bit for bit.

This file sorts last so that it runs both after every other GPU test and,
when run alone in a fresh process, with its first call doing the one-time
set-up itself (the first test calls it before any handle exists)."""
import numpy as np
import pytest

from helpers import nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
wl, m, orc = workload(), nfm(), oracle()


def assert_same_routes(got, want, what):
    """Indices equal; weights equal bit for bit (the routes are bit-exact)."""
    idx, w = got
    want_idx, want_w = want
    assert np.array_equal(idx, want_idx), f"{what}: indices differ"
    assert np.array_equal(np.asarray(w, np.float32).view(np.uint32),
                          np.asarray(want_w, np.float32).view(np.uint32)), f"{what}: weights differ"


def noalloc(lay, x, rw, bias, T, **kw):
    idx = torch.full((T, lay.top_k), -7, dtype=torch.int32, device="cuda")
    w = torch.full((T, lay.top_k), float("nan"), dtype=torch.float32, device="cuda")
    st, msg = m.router_topk_noalloc(x, rw, bias, T, lay.hidden, lay.experts, lay.top_k, idx, w,
                                    routed_scaling=lay.scaling, **kw)
    assert st == 0, msg
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


def handle_route(lay, x, T, n_group=1, topk_group=1):
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, n_group=n_group, topk_group=topk_group, max_tokens=T)
    layer.bind_layer(lay)
    idx = torch.empty((T, lay.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, lay.top_k), dtype=torch.float32, device="cuda")
    layer.route(x, T, None, idx, w)
    layer.sync()
    out = idx.cpu().numpy(), w.cpu().numpy()
    layer.close()
    return out


def device_inputs(lay, x_bits):
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    rw = torch.from_numpy(np.ascontiguousarray(lay.router_w).view(np.int16)).cuda()
    bias = torch.from_numpy(np.ascontiguousarray(lay.bias, dtype=np.float32)).cuda()
    return x, rw, bias


@pytest.mark.parametrize("cfg,tokens", [("c1", 64), ("c2", 256)])
def test_noalloc_matches_route_on_two_calls(cfg, tokens):
    """c1: the decode batch; c2: 256 prefill tokens = 16384 scores, the
    scratch's full capacity."""
    lay, x_bits = wl.config_layer(cfg)
    x_bits = x_bits[:tokens]
    T = x_bits.shape[0]
    x, rw, bias = device_inputs(lay, x_bits)
    first = noalloc(lay, x, rw, bias, T)   # before any handle: the call sets itself up
    second = noalloc(lay, x, rw, bias, T)  # a second call in a row reuses the scratch
    want = handle_route(lay, x, T)
    _, o_idx, o_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits))
    for i, got in enumerate((first, second)):
        assert_same_routes(got, want, f"call {i} vs nf_moe_route")
        assert_same_routes(got, (o_idx, o_w), f"call {i} vs oracle")


def test_noalloc_group_limited_matches_route():
    lay, x_bits = wl.config_layer("c1")
    T = x_bits.shape[0]
    x, rw, bias = device_inputs(lay, x_bits)
    got = [noalloc(lay, x, rw, bias, T, n_group=8, topk_group=4) for _ in range(2)]
    want = handle_route(lay, x, T, n_group=8, topk_group=4)
    _, o_idx, o_w = orc.route_tokens(lay, wl.bf16_bits_to_f32(x_bits), n_group=8, topk_group=4)
    for i, g in enumerate(got):
        assert_same_routes(g, want, f"group-limited call {i} vs nf_moe_route")
        assert_same_routes(g, (o_idx, o_w), f"group-limited call {i} vs oracle")


def test_noalloc_rejects_batches_beyond_the_scratch():
    lay, x_bits = wl.config_layer("c2")
    T = m.NOALLOC_MAX_SCORES // lay.experts + 1
    x, rw, bias = device_inputs(lay, x_bits[:T])
    idx = torch.full((T, lay.top_k), -7, dtype=torch.int32, device="cuda")
    w = torch.zeros((T, lay.top_k), dtype=torch.float32, device="cuda")
    st, msg = m.router_topk_noalloc(x, rw, bias, T, lay.hidden, lay.experts, lay.top_k, idx, w,
                                    routed_scaling=lay.scaling)
    assert m.NF_ERR[st] == "CAPACITY"
    assert "static scratch" in msg and str(m.NOALLOC_MAX_SCORES) in msg
    torch.cuda.synchronize()
    assert bool((idx == -7).all())  # nothing was written
