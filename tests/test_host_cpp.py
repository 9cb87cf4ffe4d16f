"""The C++ host class (host/nf_moe_layer.hpp) through its demo program: a
layer bound by checkpoint name from a tensor file and run with
TextModel::moe's host contract.  On the GPU its output must equal the Python
host path's bit for bit (same library, same inputs); without a GPU only the
program's error paths run."""
import struct
import subprocess

import numpy as np
import pytest

from helpers import MAX_ABS, MIN_COS, PKG, assert_close, nfm, workload

DEMO = PKG / "lib" / "moe_demo"
PREFIX = "model.language_model.layers.3."
KIND = {"b": np.uint16, "f": np.float32, "u": np.uint8, "8": np.uint8}


def write_nft(path, tensors: dict) -> None:
    with open(path, "wb") as f:
        f.write(b"NFT1")
        for name, (kind, arr) in tensors.items():
            a = np.array(arr, dtype=KIND[kind], order="C")  # keeps rank-0 scalars rank 0
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)) + nb + kind.encode() + struct.pack("<I", a.ndim))
            f.write(struct.pack(f"<{a.ndim}q", *a.shape) if a.ndim else b"")
            f.write(struct.pack("<Q", a.nbytes) + a.tobytes())


def layer_tensors(lay) -> dict:
    t = {PREFIX + "mlp.gate.weight": ("b", lay.router_w),
         PREFIX + "mlp.gate.e_score_correction_bias": ("f", lay.bias),
         PREFIX + "mlp.shared_experts.gate_proj.weight": ("b", lay.shared_gate),
         PREFIX + "mlp.shared_experts.up_proj.weight": ("b", lay.shared_up),
         PREFIX + "mlp.shared_experts.down_proj.weight": ("b", lay.shared_down)}
    for e in range(lay.experts):
        for proj, packed, scales, ws2, ins in (("gate_proj", lay.gate_packed, lay.gate_scales, lay.gate_ws2, lay.gate_in),
                                               ("up_proj", lay.up_packed, lay.up_scales, lay.up_ws2, lay.up_in),
                                               ("down_proj", lay.down_packed, lay.down_scales, lay.down_ws2, lay.down_in)):
            base = f"{PREFIX}mlp.experts.{e}.{proj}."
            t[base + "weight"] = ("u", packed[e])
            t[base + "weight_scale"] = ("8", scales[e])
            t[base + "weight_scale_2"] = ("f", np.float32(ws2[e]))
            t[base + "input_scale"] = ("f", np.float32(ins[e]))
    return t


def run_demo(path, out, lay, *extra):
    args = [str(DEMO), str(path), PREFIX, str(out), str(lay.hidden), str(lay.experts), str(lay.top_k), str(lay.inter),
            str(lay.shared_inter), repr(float(lay.scaling)), *extra]
    return subprocess.run(args, capture_output=True, text=True, timeout=300)


def test_demo_reports_missing_file_and_tensors(tmp_path):
    if not DEMO.exists():
        pytest.skip("demo not built")
    lay, _ = workload().config_layer("c0")
    r = run_demo(tmp_path / "none.nft", tmp_path / "y.f32", lay)
    assert r.returncode == 1 and "cannot open" in r.stderr
    write_nft(tmp_path / "x_only.nft", {"y": ("f", np.zeros((2, 2), np.float32))})
    r = run_demo(tmp_path / "x_only.nft", tmp_path / "y.f32", lay)
    assert r.returncode == 1 and "missing tensor x" in r.stderr


@pytest.mark.gpu
def test_demo_matches_python_host_path(tmp_path):
    wl = workload()
    lay, x_bits = wl.config_layer("c0")
    x = wl.bf16_bits_to_f32(x_bits)
    t = layer_tensors(lay)
    t["x"] = ("f", x)
    write_nft(tmp_path / "c0.nft", t)
    r = run_demo(tmp_path / "c0.nft", tmp_path / "y.f32", lay)
    assert r.returncode == 0, r.stderr
    y_cpp = np.fromfile(tmp_path / "y.f32", dtype=np.float32).reshape(x.shape)
    m = nfm()
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=x.shape[0])
    layer.bind_layer(lay)
    y_py = layer.forward_host(x)
    layer.close()
    assert np.array_equal(y_cpp.view(np.uint32), y_py.view(np.uint32))
    g = np.load(PKG.parent / "tests" / "golden" / "c0_reference.npz")  # the reference's own layer output
    assert_close(y_cpp, g["nvfp4_y"], MAX_ABS, MIN_COS, "C++ host vs reference")


@pytest.mark.gpu
def test_demo_missing_expert_tensor_names_it(tmp_path):
    wl = workload()
    lay, x_bits = wl.config_layer("c0")
    t = layer_tensors(lay)
    del t[PREFIX + "mlp.experts.5.up_proj.weight_scale"]
    t["x"] = ("f", wl.bf16_bits_to_f32(x_bits))
    write_nft(tmp_path / "c0.nft", t)
    r = run_demo(tmp_path / "c0.nft", tmp_path / "y.f32", lay)
    assert r.returncode == 1 and f"missing tensor {PREFIX}mlp.experts.5.up_proj.weight_scale" in r.stderr
