"""The C-ABI library loads, exports every entry point include/nf_moe.h
declares, and rejects bad descriptors before touching a device.  No compute
call runs here (there is no GPU in the CPU suite)."""
import ctypes
import re
from pathlib import Path

import pytest

from helpers import REPO, nfm

HEADER = REPO / "include" / "nf_moe.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"NF_API\s+[\w\s\*]+?\b(nf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "nf_moe_forward" in syms and "nf_moe_bind_nvfp4" in syms and len(syms) >= 16


def test_library_exports_every_declared_symbol():
    m = nfm()
    lib = m.load()
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in nf_moe.h but not exported"
    assert set(m.EXPORTED) <= set(declared_symbols())


def test_status_strings():
    lib = nfm().load()
    assert lib.nf_status_string(0) == b"ok"
    assert lib.nf_status_string(10) == b"token capacity exceeded"
    assert lib.nf_status_string(999) == b"unknown status"


def test_create_rejects_bad_descriptors_without_gpu():
    m = nfm()
    lib = m.load()
    cases = [
        dict(hidden=100),          # not a multiple of 256
        dict(inter=96),            # not a multiple of 128
        dict(top_k=0),
        dict(top_k=9, experts=8),
        dict(experts=2000),
        dict(max_tokens=0),
        dict(n_group=3),           # does not divide the experts
        dict(expert_kind=7),
    ]
    base = dict(hidden=256, experts=8, top_k=2, inter=128, shared_inter=128, n_group=1, topk_group=1, normalize=1,
                routed_scaling=1.0, swiglu_limit=10.0, expert_kind=0, max_tokens=16)
    for c in cases:
        d = m.Desc(**{**base, **c})
        h = ctypes.c_void_p()
        st = lib.nf_moe_create(ctypes.byref(d), 0, ctypes.byref(h))
        assert st != 0 and not h.value
        assert lib.nf_moe_last_error(None)
    # null arguments
    assert lib.nf_moe_create(None, 0, None) == 1
    assert lib.nf_moe_forward(None, None, None, 0, None, None, None, None) == 1
    assert lib.nf_moe_bind_nvfp4(None, 0, 0, None, None, 1.0, 1.0, 1, 16) == 1


def test_python_layer_raises_with_message_without_gpu():
    m = nfm()
    with pytest.raises(RuntimeError):
        m.MoeLayer(hidden=100, experts=8, top_k=2, inter=128, shared_inter=128)


def test_dense_and_ep_queries_without_gpu():
    """The dense MLP's create rejects shapes the GEMMs cannot tile before any
    device call, and the EP transport query answers for a NULL handle."""
    m = nfm()
    lib = m.load()
    h = ctypes.c_void_p()
    for hidden, inter, max_tokens in ((100, 512, 8), (256, 96, 8), (256, 512, 0)):
        st = lib.nf_moe_create_dense(hidden, inter, 10.0, max_tokens, 0, ctypes.byref(h))
        assert st != 0 and not h.value
        assert lib.nf_moe_last_error(None)
    assert lib.nf_moe_create_dense(256, 512, 10.0, 8, 0, None) == 1
    assert lib.nf_moe_ep_transport(None) == 0
    with pytest.raises(RuntimeError):
        m.DenseMlp(256, 100)


def test_device_buffer_checks_without_gpu():
    """forward and route take CUDA tensors on the handle's device with the
    documented dtypes, contiguous and large enough; anything else is refused
    on the host before a kernel could read or write out of bounds."""
    import numpy as np
    import torch

    m = nfm()
    f32 = ("torch.float32",)
    with pytest.raises(m.NfError, match="host array"):
        m._dev(np.zeros(4, np.float32), 4, f32, "y", 0)
    with pytest.raises(m.NfError, match="not on cuda:0"):
        m._dev(torch.zeros(4), 4, f32, "y", 0)

    class FakeCuda:
        """Duck-typed stand-in for a CUDA tensor (no GPU here)."""

        def __init__(self, n, dtype="torch.float32", contiguous=True, index=0):
            self.is_cuda, self.dtype, self.n, self.c = True, dtype, n, contiguous
            self.device = type("D", (), {"index": index})()

        def is_contiguous(self):
            return self.c

        def numel(self):
            return self.n

        def data_ptr(self):
            return 4096

    assert m._dev(FakeCuda(8), 8, f32, "y", 0) == 4096
    assert m._dev(None, 8, f32, "y", 0) is None and m._dev(1024, 8, f32, "y", 0) == 1024
    with pytest.raises(m.NfError, match="not on cuda:1"):
        m._dev(FakeCuda(8), 8, f32, "y", 1)
    with pytest.raises(m.NfError, match="dtype"):
        m._dev(FakeCuda(8, "torch.float16"), 8, f32, "y", 0)
    with pytest.raises(m.NfError, match="contiguous"):
        m._dev(FakeCuda(8, contiguous=False), 8, f32, "y", 0)
    with pytest.raises(m.NfError, match="7 elements; 8 needed"):
        m._dev(FakeCuda(7), 8, f32, "y", 0)
    assert m._dev(FakeCuda(8, "torch.int16"), 8, m._X_DTYPES, "x", 0) == 4096


def test_noalloc_wrapper_checks_buffers_before_the_library():
    """router_topk_noalloc refuses host arrays, CPU tensors, wrong dtypes and
    short buffers on the host: the library is never called (a host pointer
    would reach the router's bulk copies as a device address)."""
    import numpy as np
    import torch

    m = nfm()
    calls = []

    class Spy:
        def nf_router_topk_noalloc(self, *a):
            calls.append(a)
            return 0

    real = m._lib
    m._lib = Spy()
    try:
        T, H, E, K = 4, 256, 8, 2
        x = np.zeros((T, H), np.uint16)
        with pytest.raises(m.NfError, match="x is a host array"):
            m.router_topk_noalloc(x, 4096, 8192, T, H, E, K, 12288, 16384)
        with pytest.raises(m.NfError, match="bias is a host array"):
            m.router_topk_noalloc(1024, 4096, np.zeros(E, np.float32), T, H, E, K, 12288, 16384)
        with pytest.raises(m.NfError, match="w is not a CUDA tensor"):
            m.router_topk_noalloc(1024, 4096, 8192, T, H, E, K, 12288, torch.zeros((T, K)))

        class FakeCuda:
            def __init__(self, n, dtype):
                self.is_cuda, self.dtype, self.n = True, dtype, n
                self.device = type("D", (), {"index": 0})()

            def is_contiguous(self):
                return True

            def numel(self):
                return self.n

            def data_ptr(self):
                return 1 << 20

        ok = dict(x=FakeCuda(T * H, "torch.int16"), rw=FakeCuda(E * H, "torch.int16"),
                  b=FakeCuda(E, "torch.float32"), i=FakeCuda(T * K, "torch.int32"), w=FakeCuda(T * K, "torch.float32"))
        args = lambda **kw: [{**ok, **kw}[k] for k in ("x", "rw", "b")] + [T, H, E, K] + \
            [{**ok, **kw}[k] for k in ("i", "w")]  # noqa: E731
        with pytest.raises(m.NfError, match="router_w holds"):
            m.router_topk_noalloc(*args(rw=FakeCuda(E * H - 1, "torch.int16")))
        with pytest.raises(m.NfError, match="idx has dtype"):
            m.router_topk_noalloc(*args(i=FakeCuda(T * K, "torch.int64")))
        assert not calls
        st, msg = m.router_topk_noalloc(*args())  # every check passes: the call goes through
        assert st == 0 and len(calls) == 1
    finally:
        m._lib = real


def test_format_helpers_and_binds_check_arrays_before_the_library():
    """The NVFP4 format helpers refuse host arrays and short or mistyped
    device buffers with NF_ERR_INVALID and no library call; bind_nvfp4 refuses
    code / scale arrays that linear_nvfp4 refuses (src/text_forward.cpp:
    837-843: "NVFP4 layout" for a rank other than 2, "NVFP4 shape" for scales
    that are not [rows, cols / 16]), before the library could read past a
    short scale array; forward_host refuses an x that is not [tokens, hidden]
    and a residual of another shape."""
    import numpy as np

    m = nfm()
    calls = []

    class Spy:
        def __getattr__(self, name):
            def call(*a):
                calls.append(name)
                return 0
            return call

    class FakeCuda:
        def __init__(self, n, dtype):
            self.is_cuda, self.dtype, self.n = True, dtype, n
            self.device = type("D", (), {"index": 0})()

        def is_contiguous(self):
            return True

        def numel(self):
            return self.n

        def data_ptr(self):
            return 1 << 20

    real = m._lib
    m._lib = Spy()
    real_dev = m._current_device
    m._current_device = lambda: 0  # no GPU here: the fakes claim cuda:0
    try:
        rows, cols = 4, 64
        u8 = lambda n: FakeCuda(n, "torch.uint8")  # noqa: E731
        f32 = lambda n: FakeCuda(n, "torch.float32")  # noqa: E731
        assert m.dequantize(np.zeros(rows * cols // 2, np.uint8), u8(rows * cols // 16), 1.0, rows, cols,
                            f32(rows * cols)) == 1
        assert m.dequantize(u8(rows * cols // 2), u8(rows * cols // 16 - 1), 1.0, rows, cols, f32(rows * cols)) == 1
        assert m.dequantize(u8(rows * cols // 2), u8(rows * cols // 16), 1.0, rows, cols,
                            FakeCuda(rows * cols, "torch.float16")) == 1
        assert m.quantize(f32(rows * cols), rows, cols, 1.0, u8(rows * cols // 2), u8(rows * cols // 16),
                          f32(rows * cols - 1)) == 1
        assert m.sigmoid_ref(np.zeros(8, np.float32), 8, f32(8)) == 1
        assert not calls
        assert m.dequantize(u8(rows * cols // 2), u8(rows * cols // 16), 1.0, rows, cols, f32(rows * cols)) == 0
        assert m.quantize(f32(rows * cols), rows, cols, 1.0, u8(rows * cols // 2), u8(rows * cols // 16)) == 0
        assert m.sigmoid_ref(f32(8), 8, f32(8)) == 0
        assert calls == ["nf_nvfp4_dequantize", "nf_nvfp4_quantize", "nf_sigmoid_ref"]
        calls.clear()

        H, I = 256, 128
        layer = m.MoeLayer.borrow(1234, m.Desc(H, 8, 2, I, 0, 1, 1, 1, 1.0, 10.0, m.EXPERTS_NVFP4, 4), 0)
        layer.lib = Spy()
        codes = np.zeros((I, H // 2), np.uint8)
        with pytest.raises(m.NfError, match="NVFP4 shape mlp.experts.3.up_proj") as e:
            layer.bind_nvfp4(3, m.PROJ_UP, codes, np.zeros((I, H // 16 - 1), np.uint8), 1 / 448, 1 / 6)
        assert e.value.status == 2
        with pytest.raises(m.NfError, match="NVFP4 layout mlp.experts.3.down_proj") as e:
            layer.bind_nvfp4(3, m.PROJ_DOWN, codes, np.zeros(I * H // 16, np.uint8), 1 / 448, 1 / 6)
        assert e.value.status == 3
        dense = m.DenseMlp.borrow(1234, m.Desc(H, 1, 1, I, 0, 1, 1, 1, 1.0, 10.0, m.EXPERTS_NVFP4, 4), 0)
        dense.lib = Spy()
        with pytest.raises(m.NfError, match="NVFP4 shape mlp.gate_proj"):
            dense.bind_nvfp4(0, m.PROJ_GATE, codes, np.zeros((I - 1, H // 16), np.uint8), 1 / 448, 1 / 6)
        with pytest.raises(ValueError, match=r"\[tokens, 256\]"):
            layer.forward_host(np.zeros((2, H - 16), np.float32))
        with pytest.raises(ValueError, match="residual"):
            layer.forward_host(np.zeros((2, H), np.float32), np.zeros((1, H), np.float32))
        assert not calls
        layer.bind_nvfp4(3, m.PROJ_UP, codes, np.zeros((I, H // 16), np.uint8), 1 / 448, 1 / 6)
        assert calls == ["nf_moe_bind_nvfp4"]
    finally:
        m._lib = real
        m._current_device = real_dev
