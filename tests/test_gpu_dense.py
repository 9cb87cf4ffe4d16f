"""The dense NVFP4 MLP of the first layers (TextModel::dense_mlp,
src/text_forward.cpp:909-915) on the GPU against the oracle: the down input's
codes (the quantised swiglu_clamp_bf16 output) and the layer output within the
stated tolerance (max-abs <= 2e-2, cosine >= 0.9995), with and without the
residual, on ragged batches, through the device, host and graph paths, and
the reference's error behaviour for the dense tensor names."""
import numpy as np
import pytest

from helpers import assert_close, nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
orc, wl, m = oracle(), workload(), nfm()


def make(hidden, inter, max_tokens, seed=5):
    lay = wl.make_dense_layer(hidden, inter, seed)
    mlp = m.DenseMlp(hidden, inter, swiglu_limit=lay.swiglu_limit, max_tokens=max_tokens)
    mlp.bind_layer(lay)
    return lay, mlp


def tokens(hidden, T, seed=5):
    return wl.make_tokens(dict(hidden=hidden, tokens=T), seed)


def gpu_forward(mlp, x_bits, residual=None):
    T, H = x_bits.shape
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    res = None if residual is None else torch.from_numpy(residual).cuda()
    mlp.forward(x, y, T, res)
    mlp.sync()
    return y.cpu().numpy()


# (256, 512): K too short to split; (256, 2048): the down projection split
# into K slices and reduced inside the down GEMM (tiles of <= 32 rows at
# T = 16, two ragged row blocks at T = 200; at T = 48 the gate/up tile's rows
# repeated in the upper TMEM lane quadrants, rows 48-63 of each copy empty);
# (2048, 10240): the benchmark's dense layers at the decode batch (14 K
# slices, 64 rows repeated)
@pytest.mark.parametrize("hidden,inter,T", [(256, 512, 16), (256, 2048, 16), (256, 2048, 48), (256, 2048, 200),
                                            (2048, 10240, 64)])
def test_dense_against_oracle(hidden, inter, T):
    lay, mlp = make(hidden, inter, T)
    x_bits = tokens(hidden, T)
    x = wl.bf16_bits_to_f32(x_bits)
    res = np.random.Generator(np.random.PCG64(T)).standard_normal(x.shape).astype(np.float32)
    want, h = orc.dense_mlp(orc.port(), lay, x, None, taps=True)
    got = gpu_forward(mlp, x_bits)
    assert_close(got, want, what=f"dense H{hidden} I{inter} T{T}")
    # the down GEMM's input: codes and block scales of swiglu_clamp_bf16's
    # output, quantised with down_proj's input scale (rows are the tokens in
    # order: one segment starting at row 0)
    codes = mlp.debug_read("h_codes", np.uint8, T * inter // 2).reshape(T, inter // 2)
    rows_pad = (T + 127) // 128 * 128
    sf = m.sf_from_atoms(mlp.debug_read("h_sf", np.uint8, rows_pad * inter // 16), T, inter // 16)
    _, want_codes, want_sf = orc.quant_codes(orc.port(), h, lay.down_in)
    # SiLU here differs from libm's by a few ulp, which can move a BF16
    # rounding of the activation, so a handful of codes may differ
    assert np.mean(codes != want_codes) < 1e-3
    assert np.mean(sf != want_sf) < 1e-3
    got_r = gpu_forward(mlp, x_bits, res)
    want_r = orc.dense_mlp(orc.port(), lay, x, res)
    assert_close(got_r, want_r, what=f"dense+residual H{hidden} I{inter} T{T}")
    mlp.close()


def test_dense_host_graph_and_repeat_agree():
    lay, mlp = make(256, 512, 130)
    x_bits = tokens(256, 130, seed=9)
    x = wl.bf16_bits_to_f32(x_bits)
    res = np.random.Generator(np.random.PCG64(3)).standard_normal(x.shape).astype(np.float32)
    y1 = gpu_forward(mlp, x_bits, res)
    y2 = gpu_forward(mlp, x_bits, res)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    yh = mlp.forward_host(x, res)
    assert np.array_equal(yh.view(np.uint32), y1.view(np.uint32))
    # graph replay on a dedicated stream gives the same bits
    mlp.set_graph_mode(True)
    s = torch.cuda.Stream()
    xd = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    rd = torch.from_numpy(res).cuda()
    yd = torch.empty((130, 256), dtype=torch.float32, device="cuda")
    for _ in range(3):
        mlp.forward(xd, yd, 130, rd, stream=s.cuda_stream)
    mlp.sync(s.cuda_stream)
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), y1.view(np.uint32))
    # fewer tokens than the capacity, and none
    y5 = gpu_forward(mlp, x_bits[:5], res[:5])
    assert np.array_equal(y5.view(np.uint32), y1[:5].view(np.uint32))
    mlp.forward(xd, yd, 0)
    mlp.close()


def test_dense_bind_from_store_and_errors():
    lay = wl.make_dense_layer(256, 512, 11)
    prefix = "model.language_model.layers.0."
    store = {}
    for name in ("gate", "up", "down"):
        base = f"{prefix}mlp.{name}_proj"
        store[base + ".weight"] = getattr(lay, f"{name}_packed")
        store[base + ".weight_scale"] = getattr(lay, f"{name}_scales")
        store[base + ".weight_scale_2"] = np.array(getattr(lay, f"{name}_ws2"), np.float32)
        store[base + ".input_scale"] = np.array(getattr(lay, f"{name}_in"), np.float32)
    mlp = m.DenseMlp(256, 512, max_tokens=8)
    mlp.bind_from_store(store, prefix)
    x_bits = tokens(256, 8, seed=2)
    want = orc.dense_mlp(orc.port(), lay, wl.bf16_bits_to_f32(x_bits))
    assert_close(gpu_forward(mlp, x_bits), want, what="dense bound by name")
    # a dense handle has no routes, router or bias
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = torch.empty((8, 256), dtype=torch.float32, device="cuda")
    idx = torch.empty((8, 1), dtype=torch.int32, device="cuda")
    with pytest.raises(m.NfError, match="no routes"):
        m.MoeLayer.forward(mlp, x, y, 8, None, idx, None)
    with pytest.raises(m.NfError, match="no router"):
        mlp.route(x, 8, idx_dev=idx)
    mlp.close()

    # the reference's messages, with the dense layers' tensor names
    fresh = m.DenseMlp(256, 512, max_tokens=8)
    with pytest.raises(m.NfError, match="NVFP4 shape mlp.gate_proj"):
        fresh.bind_nvfp4(0, m.PROJ_GATE, lay.down_packed, lay.down_scales, lay.gate_ws2, lay.gate_in)
    with pytest.raises(m.NfError, match="NVFP4 input scale"):
        fresh.bind_nvfp4(0, m.PROJ_UP, lay.up_packed, lay.up_scales, lay.up_ws2, float("nan"))
    with pytest.raises(m.NfError, match="holds no mlp.gate.e_score_correction_bias"):
        fresh.bind_f32(m.F32_ROUTER_BIAS, np.zeros(1, np.float32))
    fresh.bind_nvfp4(0, m.PROJ_GATE, lay.gate_packed, lay.gate_scales, lay.gate_ws2, lay.gate_in)
    fresh.bind_nvfp4(0, m.PROJ_UP, lay.up_packed, lay.up_scales, lay.up_ws2, lay.up_in)
    with pytest.raises(m.NfError, match="missing tensor mlp.down_proj"):
        fresh.finalize()
    with pytest.raises(m.NfError, match="missing tensor model.language_model.layers.0.mlp.up_proj.weight_scale_2"):
        m.DenseMlp(256, 512, max_tokens=8).bind_from_store(
            {k: v for k, v in store.items() if not k.endswith("up_proj.weight_scale_2")}, prefix)
    fresh.close()
    with pytest.raises(m.NfError):
        m.DenseMlp(256, 100)


def test_dense_against_reference_golden():
    """The GPU dense MLP against the reference's own outputs (committed golden
    file, no oracle involved), with and without the residual."""
    from pathlib import Path

    from golden.make_golden import dense_case

    g = np.load(Path(__file__).resolve().parent / "golden" / "dense_reference.npz")
    lay, x_bits, res = dense_case()
    mlp = m.DenseMlp(lay.hidden, lay.inter, swiglu_limit=lay.swiglu_limit, max_tokens=x_bits.shape[0])
    mlp.bind_layer(lay)
    assert_close(gpu_forward(mlp, x_bits), g["y"], what="dense vs reference golden")
    assert_close(gpu_forward(mlp, x_bits, res), g["y_residual"], what="dense + residual vs reference golden")
    mlp.close()


def test_dense_large_batch_wide_stages():
    """5,000 tokens, H 512, I 1280, with 512-K stages: the down projection is
    not split and both GEMMs take 512-K stages; the down GEMM's K (1280) ends
    in a half stage.
    Tokens are independent, so a subset of 97 rows checks them fully."""
    lay, mlp = make(512, 1280, 5000, seed=13)
    mlp.set_expert_gemm("wide")
    x_bits = tokens(512, 5000, seed=13)
    got = gpu_forward(mlp, x_bits)
    sel = np.arange(0, 5000, 52)
    want = orc.dense_mlp(orc.port(), lay, wl.bf16_bits_to_f32(x_bits[sel]), None)
    assert_close(got[sel], want, what="dense H512 I1280 T5000 (512-K stages)")
    mlp.close()
