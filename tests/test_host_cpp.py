"""The C++ host class (host/nf_moe_layer.hpp) through its demo program: a
layer bound by checkpoint name from a tensor file and run with
TextModel::moe's host contract.  On the GPU its output must equal the Python
host path's bit for bit (same library, same inputs); without a GPU only the
program's error paths run."""
import struct
import subprocess

import numpy as np
import pytest

from helpers import MAX_ABS, MIN_COS, PKG, assert_close, load_module, nfm, workload

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
def test_demo_expert_parallel_matches_one_gpu(tmp_path):
    """The C++ host class's expert-parallel constructor and host-buffer
    forward on two GPUs (two processes, the group id handed over in a file):
    each rank's share of the rows equals the one-GPU run bit for bit."""
    import os

    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    wl = workload()
    lay, x_bits = wl.config_layer("c0")
    x = wl.bf16_bits_to_f32(x_bits)
    t = layer_tensors(lay)
    t["x"] = ("f", x)
    write_nft(tmp_path / "c0.nft", t)
    r = run_demo(tmp_path / "c0.nft", tmp_path / "y1.f32", lay)
    assert r.returncode == 0, r.stderr
    y1 = np.fromfile(tmp_path / "y1.f32", dtype=np.float32).reshape(x.shape)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    args = [str(DEMO), str(tmp_path / "c0.nft"), PREFIX, "", str(lay.hidden), str(lay.experts), str(lay.top_k),
            str(lay.inter), str(lay.shared_inter), repr(float(lay.scaling))]
    procs = []
    for rank in range(2):
        a = list(args)
        a[3] = str(tmp_path / f"y_rank{rank}.f32")
        a += [str(rank), "--ep", str(rank), "2", str(tmp_path / "group.id")]
        procs.append(subprocess.Popen(a, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env))
    outs = [p.communicate(timeout=300) for p in procs]
    for p, (out, err) in zip(procs, outs):
        assert p.returncode == 0, err
    T, H = x.shape
    parts = [np.fromfile(tmp_path / f"y_rank{rank}.f32", dtype=np.float32) for rank in range(2)]
    y2 = np.concatenate(parts).reshape(T, H)
    assert np.array_equal(y2.view(np.uint32), y1.view(np.uint32))


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


@pytest.mark.gpu
def test_demo_refuses_scales_of_the_wrong_rank_or_shape(tmp_path):
    """linear_nvfp4's checks (src/text_forward.cpp:837-843) by checkpoint name:
    a weight_scale that is not rank 2 is "NVFP4 layout <name>", one that is not
    [N, K/16] for codes [N, K/2] is "NVFP4 shape <name>" (the library would
    otherwise read N K/16 bytes past a shorter tensor)."""
    wl = workload()
    lay, x_bits = wl.config_layer("c0")
    name = f"{PREFIX}mlp.experts.2.down_proj"
    for scales, msg in ((lay.down_scales[2].ravel(), "NVFP4 layout"), (lay.down_scales[2][:, :-1], "NVFP4 shape"),
                        (lay.down_scales[2][:-1], "NVFP4 shape")):
        t = layer_tensors(lay)
        t[name + ".weight_scale"] = ("8", scales)
        t["x"] = ("f", wl.bf16_bits_to_f32(x_bits))
        write_nft(tmp_path / "c0.nft", t)
        r = run_demo(tmp_path / "c0.nft", tmp_path / "y.f32", lay)
        assert r.returncode == 1 and f"{msg} {name}" in r.stderr, r.stderr


# ---- safetensors checkpoints (host/nf_safetensors.hpp, nf_moe.safetensors_store)
ST_DTYPE = {"b": "BF16", "f": "F32", "u": "U8", "8": "F8_E4M3"}


def write_safetensors(path, tensors: dict, header_patch=None) -> None:
    """One safetensors shard: u64 header length, JSON header, packed data."""
    import json

    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, (kind, arr) in tensors.items():
        a = np.array(arr, dtype=KIND[kind], order="C")
        header[name] = {"dtype": ST_DTYPE[kind], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    if header_patch:
        header_patch(header)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def write_checkpoint(directory, tensors: dict, shards: int = 2) -> None:
    """A checkpoint directory: the tensors spread over `shards` files and a
    model.safetensors.index.json weight map."""
    import json

    directory.mkdir(parents=True, exist_ok=True)
    names = list(tensors)
    parts = [names[i::shards] for i in range(shards)]
    wmap = {}
    for i, part in enumerate(parts):
        fname = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(directory / fname, {n: tensors[n] for n in part})
        wmap.update({n: fname for n in part})
    (directory / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wmap}))


def dense_tensors(lay, prefix) -> dict:
    t = {}
    for name in ("gate", "up", "down"):
        base = f"{prefix}mlp.{name}_proj."
        t[base + "weight"] = ("u", getattr(lay, f"{name}_packed"))
        t[base + "weight_scale"] = ("8", getattr(lay, f"{name}_scales"))
        t[base + "weight_scale_2"] = ("f", np.float32(getattr(lay, f"{name}_ws2")))
        t[base + "input_scale"] = ("f", np.float32(getattr(lay, f"{name}_in")))
    return t


def test_safetensors_store_errors(tmp_path):
    """The checkpoint store's failures, from the C++ demo (before any device
    work) and from the Python reader, with the reference Store's messages."""
    m = nfm()
    lay, _ = workload().config_layer("c0")
    cases = []
    empty = tmp_path / "empty"
    empty.mkdir()
    cases.append((empty, "missing model.safetensors.index.json"))
    bad = tmp_path / "bad"
    bad.mkdir()
    (bad / "model.safetensors").write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    cases.append((bad, "bad safetensors header"))
    dt = tmp_path / "dtype"
    dt.mkdir()
    write_safetensors(dt / "model.safetensors", {"x": ("f", np.zeros((2, 4), np.float32))},
                      lambda h: h["x"].update(dtype="F16"))
    cases.append((dt, "unsupported dtype F16 for x"))
    rng = tmp_path / "range"
    rng.mkdir()
    write_safetensors(rng / "model.safetensors", {"x": ("f", np.zeros((2, 4), np.float32))},
                      lambda h: h["x"].update(data_offsets=[0, 4096]))
    cases.append((rng, "tensor data out of range for x"))
    size = tmp_path / "size"
    size.mkdir()
    write_safetensors(size / "model.safetensors", {"x": ("f", np.zeros((2, 4), np.float32))},
                      lambda h: h["x"].update(shape=[2, 3]))
    cases.append((size, "tensor size mismatch for x"))
    # an element count whose byte size wraps a 64-bit product (2^62 F32 in
    # zero bytes), one past any shard, a negative shape, a bad \u escape
    for tag, patch, msg in (("wrap", dict(shape=[1 << 31, 1 << 31], data_offsets=[0, 0]), "tensor size mismatch for x"),
                            ("huge", dict(shape=[1 << 32, 1 << 32], data_offsets=[0, 0]), "tensor size mismatch for x"),
                            ("neg", dict(shape=[-2, -4]), "negative dimension for x")):
        d = tmp_path / tag
        d.mkdir()
        write_safetensors(d / "model.safetensors", {"x": ("f", np.zeros((2, 4), np.float32))},
                          lambda h, patch=patch: h["x"].update(**patch))
        cases.append((d, msg))
    esc = tmp_path / "escape"
    esc.mkdir()
    h = b'{"x\\uZZZZ":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}'
    (esc / "model.safetensors").write_bytes(struct.pack("<Q", len(h)) + h + bytes(4))
    cases.append((esc, "bad safetensors header"))
    shard = tmp_path / "shard"
    write_checkpoint(shard, {"x": ("f", np.zeros((2, 4), np.float32)), "y": ("f", np.zeros(3, np.float32))})
    (shard / "model-00002-of-00002.safetensors").unlink()
    cases.append((shard, "cannot open shard"))
    nox = tmp_path / "nox"
    write_checkpoint(nox, {"y": ("f", np.zeros(3, np.float32))}, shards=1)
    for d, msg in cases + [(nox, None)]:
        if msg is not None:
            with pytest.raises(m.NfError, match=msg):
                m.safetensors_store(d)
        if DEMO.exists():
            r = run_demo(d, tmp_path / "y.f32", lay)
            assert r.returncode == 1 and (msg or "missing tensor x") in r.stderr, r.stderr


def test_safetensors_store_reads_checkpoint(tmp_path):
    """Every tensor of a two-shard checkpoint comes back with its name, kind,
    shape and bytes (rank-0 scalars stay rank 0)."""
    m = nfm()
    lay, x_bits = workload().config_layer("c0")
    t = layer_tensors(lay)
    write_checkpoint(tmp_path / "ckpt", t)
    store = m.safetensors_store(tmp_path / "ckpt")
    assert set(store) == set(t)
    for name, (kind, arr) in t.items():
        a = np.asarray(arr, dtype=KIND[kind])
        assert store[name].dtype == a.dtype and store[name].shape == a.shape
        assert np.array_equal(store[name], a)


@pytest.mark.gpu
def test_checkpoint_directory_binds_moe_and_dense(tmp_path):
    """Checkpoint -> device residency: a MoE layer and a dense MLP bound by
    name from safetensors shards (C++ store in the demo, Python store in
    MoeLayer / DenseMlp.bind_from_store) give the same bits as binding the
    arrays directly."""
    wl, m = workload(), nfm()
    lay, x_bits = wl.config_layer("c0")
    x = wl.bf16_bits_to_f32(x_bits)
    t = layer_tensors(lay)
    t["x"] = ("f", x)
    write_checkpoint(tmp_path / "moe", t, shards=3)
    r = run_demo(tmp_path / "moe", tmp_path / "y.f32", lay)
    assert r.returncode == 0, r.stderr
    y_cpp = np.fromfile(tmp_path / "y.f32", dtype=np.float32).reshape(x.shape)
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=x.shape[0])
    layer.bind_layer(lay)
    y_ref = layer.forward_host(x)
    layer.close()
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=x.shape[0])
    layer.bind_from_store(m.safetensors_store(tmp_path / "moe"), PREFIX)
    y_py = layer.forward_host(x)
    layer.close()
    assert np.array_equal(y_cpp.view(np.uint32), y_ref.view(np.uint32))
    assert np.array_equal(y_py.view(np.uint32), y_ref.view(np.uint32))

    dl = wl.make_dense_layer(256, 512, 21)
    dprefix = "model.language_model.layers.0."
    xd = wl.bf16_bits_to_f32(wl.make_tokens(dict(hidden=256, tokens=12), 21))
    td = dense_tensors(dl, dprefix)
    td["x"] = ("f", xd)
    write_checkpoint(tmp_path / "dense", td)
    r = subprocess.run([str(DEMO), str(tmp_path / "dense"), dprefix, str(tmp_path / "yd.f32"), "256", "0", "1", "512",
                        "0", "1.0"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    yd_cpp = np.fromfile(tmp_path / "yd.f32", dtype=np.float32).reshape(xd.shape)
    mlp = m.DenseMlp(256, 512, max_tokens=12)
    mlp.bind_layer(dl)
    yd_ref = mlp.forward_host(xd)
    mlp.close()
    assert np.array_equal(yd_cpp.view(np.uint32), yd_ref.view(np.uint32))
    orc = load_module("nf_oracle_py", PKG.parent / "oracle" / "oracle.py")
    assert_close(yd_cpp, orc.dense_mlp(orc.port(), dl, xd), MAX_ABS, MIN_COS, "dense from checkpoint vs oracle")
