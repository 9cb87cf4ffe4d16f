"""ctypes access to the CPU checkers (TEST INFRASTRUCTURE ONLY).

  port()  -> _build/libnf_oracle.so, the plain-C restatement (nf_oracle.c)
  ref()   -> _ref/libnf_ref.so, the reference's own sources (ref_shim.cpp),
             or None when they were not built (no reference tree)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module, and only to check or time the CPU path, never as the product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "libnf_oracle.so"
REF_LIB = HERE / "_ref" / "libnf_ref.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_I64 = ctypes.c_int64


class MoeWeights(ctypes.Structure):
    _fields_ = [
        ("hidden", _I), ("experts", _I), ("top_k", _I), ("inter", _I), ("shared_inter", _I),
        ("scaling", _F), ("swiglu_limit", _F),
        ("n_group", _I), ("topk_group", _I), ("normalize", _I), ("bf16_experts", _I),
        ("router_w", _P), ("router_bias", _P),
        ("gate_packed", _P), ("gate_scales", _P), ("up_packed", _P), ("up_scales", _P),
        ("down_packed", _P), ("down_scales", _P),
        ("gate_ws2", _P), ("gate_in", _P), ("up_ws2", _P), ("up_in", _P), ("down_ws2", _P), ("down_in", _P),
        ("gate_bf16", _P), ("up_bf16", _P), ("down_bf16", _P),
        ("shared_gate", _P), ("shared_up", _P), ("shared_down", _P),
    ]


class DenseWeights(ctypes.Structure):
    _fields_ = [
        ("hidden", _I), ("inter", _I), ("swiglu_limit", _F),
        ("gate_packed", _P), ("gate_scales", _P), ("up_packed", _P), ("up_scales", _P),
        ("down_packed", _P), ("down_scales", _P),
        ("gate_ws2", _F), ("gate_in", _F), ("up_ws2", _F), ("up_in", _F), ("down_ws2", _F), ("down_in", _F),
    ]


def build() -> None:
    """Builds the checker libraries (the reference one only when its tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_port = None
_ref = None


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            build()
        lib = ctypes.CDLL(str(PORT_LIB))
        lib.or_bf16_to_f32.restype = _F
        lib.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
        lib.or_f32_to_bf16.restype = ctypes.c_uint16
        lib.or_f32_to_bf16.argtypes = [_F]
        lib.or_f32_to_e4m3.restype = ctypes.c_uint8
        lib.or_f32_to_e4m3.argtypes = [_F]
        lib.or_e4m3_to_f32.restype = _F
        lib.or_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        lib.or_e2m1.restype = _F
        lib.or_e2m1.argtypes = [ctypes.c_uint8]
        lib.or_cast_to_e2m1.restype = _F
        lib.or_cast_to_e2m1.argtypes = [_F]
        lib.or_e2m1_code.restype = ctypes.c_uint8
        lib.or_e2m1_code.argtypes = [_F]
        lib.or_sigmoid.restype = _F
        lib.or_sigmoid.argtypes = [_F]
        lib.or_quant_nvfp4_activation.restype = _I
        lib.or_quant_nvfp4_activation.argtypes = [_P, _I, _F, _P, _P, _P]
        lib.or_gemv_nvfp4_rows.restype = None
        lib.or_gemv_nvfp4_rows.argtypes = [_P, _P, _F, _F, _P, _I, _I, _I, _I, _P]
        lib.or_gemv_bf16.restype = None
        lib.or_gemv_bf16.argtypes = [_P, _P, _I, _I, _I, _I, _P]
        lib.or_linear_nvfp4.restype = _I
        lib.or_linear_nvfp4.argtypes = [_P, _P, _F, _F, _P, _I, _P, _I]
        lib.or_router_select.restype = None
        lib.or_router_select.argtypes = [_P, _P, _I, _I, _F, _I, _P, _P]
        lib.or_router_select_grouped.restype = None
        lib.or_router_select_grouped.argtypes = [_P, _P, _I, _I, _F, _I, _I, _I, _P, _P]
        lib.or_swiglu_clamp.restype = None
        lib.or_swiglu_clamp.argtypes = [_P, _P, _I, _F, _P]
        lib.or_swiglu_clamp_bf16.restype = None
        lib.or_swiglu_clamp_bf16.argtypes = [_P, _P, _I, _F, _P]
        lib.or_mhc_combine.restype = None
        lib.or_mhc_combine.argtypes = [_P, _P, _P, _P, _I, _I, _P]
        lib.or_nvfp4_dequantize.restype = _I
        lib.or_nvfp4_dequantize.argtypes = [_P, _P, _F, _I64, _I64, _P]
        lib.or_rmsnorm.restype = None
        lib.or_rmsnorm.argtypes = [_P, _P, _F, _I, _P]
        lib.or_dense_residual_proj.restype = None
        lib.or_dense_residual_proj.argtypes = [_P, _P, _P, _F, _I, _P]
        lib.or_moe_layer.restype = _I
        lib.or_moe_layer.argtypes = [ctypes.POINTER(MoeWeights), _I, _P, _P, _P, _P, _P, _P, _P]
        lib.or_expert_forward.restype = _I
        lib.or_expert_forward.argtypes = [ctypes.POINTER(MoeWeights), _I, _P, _P, _P]
        lib.or_router_logits.restype = None
        lib.or_router_logits.argtypes = [ctypes.POINTER(MoeWeights), _P, _P]
        lib.or_route_tokens.restype = None
        lib.or_route_tokens.argtypes = [ctypes.POINTER(MoeWeights), _I, _P, _P, _P, _P]
        lib.or_sigmoid_array.restype = None
        lib.or_sigmoid_array.argtypes = [_P, _I64, _P]
        lib.or_dense_mlp.restype = _I
        lib.or_dense_mlp.argtypes = [ctypes.POINTER(DenseWeights), _I, _P, _P, _P, _P]
        _port = lib
    return _port


def ref() -> ctypes.CDLL | None:
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            return None
        lib = ctypes.CDLL(str(REF_LIB))
        lib.ref_sigmoid.restype = _F
        lib.ref_sigmoid.argtypes = [_F]
        lib.ref_f32_to_e4m3.restype = ctypes.c_uint8
        lib.ref_f32_to_e4m3.argtypes = [_F]
        lib.ref_e4m3_to_f32.restype = _F
        lib.ref_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        lib.ref_e2m1.restype = _F
        lib.ref_e2m1.argtypes = [ctypes.c_uint8]
        lib.ref_cast_to_e2m1.restype = _F
        lib.ref_cast_to_e2m1.argtypes = [_F]
        lib.ref_f32_to_bf16.restype = ctypes.c_uint16
        lib.ref_f32_to_bf16.argtypes = [_F]
        lib.ref_quant_dequant.restype = _I
        lib.ref_quant_dequant.argtypes = [_P, _I, _F, _P]
        lib.ref_gemv_nvfp4_rows.restype = None
        lib.ref_gemv_nvfp4_rows.argtypes = [_P, _P, _F, _F, _P, _I, _I, _I, _I, _P]
        lib.ref_gemv_bf16.restype = None
        lib.ref_gemv_bf16.argtypes = [_P, _P, _I, _I, _I, _I, _P]
        lib.ref_router_select.restype = None
        lib.ref_router_select.argtypes = [_P, _P, _I, _I, _F, _I, _P, _P]
        lib.ref_swiglu_clamp.restype = None
        lib.ref_swiglu_clamp.argtypes = [_P, _P, _I, _F, _P]
        lib.ref_swiglu_clamp_bf16.restype = None
        lib.ref_swiglu_clamp_bf16.argtypes = [_P, _P, _I, _F, _P]
        lib.ref_mhc_combine.restype = None
        lib.ref_mhc_combine.argtypes = [_P, _P, _P, _P, _I, _I, _P]
        lib.ref_nvfp4_dequantize.restype = _I
        lib.ref_nvfp4_dequantize.argtypes = [_P, _I64, _P, _I64, _F, _I64, _I64, _P, _I64]
        lib.ref_dense_residual_proj.restype = None
        lib.ref_dense_residual_proj.argtypes = [_P, _P, _P, _F, _I, _P]
        lib.ref_rmsnorm.restype = None
        lib.ref_rmsnorm.argtypes = [_P, _P, _F, _I, _P]
        lib.ref_moe_layer.restype = _I
        lib.ref_moe_layer.argtypes = [ctypes.POINTER(MoeWeights), _I, _P, _P, _P, _P, _P]
        lib.ref_dense_mlp.restype = _I
        lib.ref_dense_mlp.argtypes = [ctypes.POINTER(DenseWeights), _I, _P, _P, _P]
        _ref = lib
    return _ref


def p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be contiguous"
    return a.ctypes.data


def weights_struct(lay, n_group: int = 1, topk_group: int = 1, normalize: bool = True) -> tuple[MoeWeights, list]:
    """MoeWeights over a workload.Layer (keeps the arrays alive in `keep`)."""
    keep = []

    def c(a, dt):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a.ctypes.data

    w = MoeWeights()
    w.hidden, w.experts, w.top_k, w.inter, w.shared_inter = lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter
    w.scaling, w.swiglu_limit = lay.scaling, lay.swiglu_limit
    w.n_group, w.topk_group, w.normalize, w.bf16_experts = n_group, topk_group, int(normalize), int(lay.bf16_experts)
    w.router_w = c(lay.router_w, np.uint16)
    w.router_bias = c(lay.bias, np.float32)
    for name in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
        setattr(w, name, c(getattr(lay, name), np.uint8))
    for name in ("gate_ws2", "gate_in", "up_ws2", "up_in", "down_ws2", "down_in"):
        setattr(w, name, c(getattr(lay, name), np.float32))
    for name in ("gate_bf16", "up_bf16", "down_bf16", "shared_gate", "shared_up", "shared_down"):
        setattr(w, name, c(getattr(lay, name), np.uint16))
    return w, keep


def moe_layer(lib, lay, x_f32: np.ndarray, residual: np.ndarray | None = None, n_group: int = 1,
              topk_group: int = 1, taps: bool = False):
    """Runs or_moe_layer (port) or ref_moe_layer (reference) on fp32 rows.
    Returns y, indices, weights (and routed / shared taps for the port)."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    T = x.shape[0]
    y = np.zeros_like(x)
    idx = np.zeros((T, lay.top_k), np.int32)
    wt = np.zeros((T, lay.top_k), np.float32)
    res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
    ws, keep = weights_struct(lay, n_group, topk_group)
    if hasattr(lib, "or_moe_layer"):
        routed = np.zeros_like(x) if taps else None
        shared = np.zeros_like(x) if taps else None
        rc = lib.or_moe_layer(ctypes.byref(ws), T, p(x), p(res), p(y), p(idx), p(wt), p(routed), p(shared))
        if rc != 0:
            raise RuntimeError("oracle rejected the layer (NVFP4 input scale)")
        return (y, idx, wt, routed, shared) if taps else (y, idx, wt)
    rc = lib.ref_moe_layer(ctypes.byref(ws), T, p(x), p(res), p(y), p(idx), p(wt))
    if rc != 0:
        raise RuntimeError(f"reference moe composition failed ({rc})")
    del keep
    return y, idx, wt


def quant_codes(lib, x: np.ndarray, input_scale: float):
    """or_quant_nvfp4_activation over rows: (fake-quant values, packed codes, scale codes)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    y = np.zeros_like(x)
    codes = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, cols // 16), np.uint8)
    for r in range(rows):
        rc = lib.or_quant_nvfp4_activation(p(x[r]), cols, input_scale, p(y[r]), p(codes[r]), p(scales[r]))
        if rc != 0:
            raise RuntimeError("NVFP4 input scale")
    return y, codes, scales


def route_tokens(lay, x_f32: np.ndarray, n_group: int = 1, topk_group: int = 1):
    """Port router over T tokens: (logits [T, E], indices [T, k], weights [T, k])."""
    lib = port()
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    T = x.shape[0]
    logits = np.zeros((T, lay.experts), np.float32)
    idx = np.zeros((T, lay.top_k), np.int32)
    wt = np.zeros((T, lay.top_k), np.float32)
    ws, keep = weights_struct(lay, n_group, topk_group)
    lib.or_route_tokens(ctypes.byref(ws), T, p(x), p(logits), p(idx), p(wt))
    del keep
    return logits, idx, wt


def sigmoid_array(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    port().or_sigmoid_array(p(x), x.size, p(y))
    return y


def expert_forward(lay, e: int, x_f32: np.ndarray):
    """(h [I], down [H]) of expert e for one token (port)."""
    lib = port()
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    h = np.zeros(lay.inter, np.float32)
    d = np.zeros(lay.hidden, np.float32)
    ws, keep = weights_struct(lay)
    rc = lib.or_expert_forward(ctypes.byref(ws), e, p(x), p(h), p(d))
    del keep
    if rc != 0:
        raise RuntimeError("NVFP4 input scale")
    return h, d


def dense_struct(lay) -> tuple[DenseWeights, list]:
    """DenseWeights over a workload.DenseLayer (keeps the arrays alive in `keep`)."""
    keep = []
    w = DenseWeights()
    w.hidden, w.inter, w.swiglu_limit = lay.hidden, lay.inter, lay.swiglu_limit
    for name in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
        a = np.ascontiguousarray(getattr(lay, name), dtype=np.uint8)
        keep.append(a)
        setattr(w, name, a.ctypes.data)
    for name in ("gate_ws2", "gate_in", "up_ws2", "up_in", "down_ws2", "down_in"):
        setattr(w, name, float(getattr(lay, name)))
    return w, keep


def dense_mlp(lib, lay, x_f32: np.ndarray, residual: np.ndarray | None = None, taps: bool = False):
    """or_dense_mlp (port) or ref_dense_mlp (reference) on fp32 rows: y, and
    with taps (port only) also swiglu_clamp_bf16's output h [T, I]."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    T = x.shape[0]
    y = np.zeros_like(x)
    res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
    ws, keep = dense_struct(lay)
    if hasattr(lib, "or_dense_mlp"):
        h = np.zeros((T, lay.inter), np.float32) if taps else None
        rc = lib.or_dense_mlp(ctypes.byref(ws), T, p(x), p(res), p(y), p(h))
        if rc != 0:
            raise RuntimeError("oracle rejected the dense MLP (NVFP4 input scale)")
        return (y, h) if taps else y
    rc = lib.ref_dense_mlp(ctypes.byref(ws), T, p(x), p(res), p(y))
    del keep
    if rc != 0:
        raise RuntimeError(f"reference dense_mlp composition failed ({rc})")
    return y
