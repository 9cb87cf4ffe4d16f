"""Python host binding of libnf_moe.so (include/nf_moe.h) through ctypes.

`MoeLayer` mirrors the reference's MoE contract: weights are bound by their
checkpoint names (parameter_schema, src/parameter_schema.cpp:53-98) from a
name -> array mapping (the role of the reference's safetensors Store,
src/text_forward.cpp:328-495), and `forward` runs TextModel::moe
(src/text_forward.cpp:924-963) for a batch of tokens.  Failures raise
RuntimeError carrying the library's message, the way the reference's
fail() throws std::runtime_error (src/text_forward.cpp:40).

There is no fallback: if the CUDA library is missing or cannot load, this
module raises.  Device buffers are passed as raw pointers (torch tensors'
data_ptr() or integers); torch is only used by callers for device memory.
"""
from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path
from typing import Mapping

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libnf_moe.so"

NF_OK = 0
NF_ERR = {1: "INVALID", 2: "SHAPE", 3: "LAYOUT", 4: "SCALE", 5: "STATE", 6: "CUDA", 7: "TIMEOUT",
          8: "UNSUPPORTED", 9: "NOMEM", 10: "CAPACITY"}
PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2
_PROJ_NAMES = {PROJ_GATE: "gate_proj", PROJ_UP: "up_proj", PROJ_DOWN: "down_proj"}
BF16_ROUTER, BF16_SHARED_GATE, BF16_SHARED_UP, BF16_SHARED_DOWN = 0, 1, 2, 3
BF16_EXPERT_GATE, BF16_EXPERT_UP, BF16_EXPERT_DOWN = 4, 5, 6
F32_ROUTER_BIAS = 0
EXPERTS_NVFP4, EXPERTS_BF16 = 0, 1
EXPERT_GEMM = dict(one_sm=0, wide=1, pair=2)  # nf_moe_set_expert_gemm (NF_GEMM_*)
DBG = dict(counts=0, seg_offset=1, pair_row=2, row_token=3, act_codes=4, act_sf=5, h_codes=6, h_sf=7, down=8,
           shared=9, rows=10, logits=11, screen_count=12)

EXPORTED = [
    "nf_moe_create", "nf_moe_destroy", "nf_moe_last_error", "nf_status_string", "nf_moe_bind_nvfp4",
    "nf_moe_bind_bf16", "nf_moe_bind_f32", "nf_moe_finalize", "nf_moe_forward", "nf_moe_forward_host",
    "nf_moe_sync", "nf_moe_route", "nf_moe_debug_tensor", "nf_moe_debug_read", "nf_nvfp4_dequantize", "nf_nvfp4_quantize",
    "nf_sigmoid_ref", "nf_moe_profile", "nf_moe_stage_times", "nf_format_selfcheck", "nf_moe_set_graph_mode", "nf_moe_set_expert_gemm",
    "nf_router_topk_noalloc", "nf_ep_unique_id", "nf_moe_create_ep", "nf_moe_create_ep_replicated", "nf_moe_create_dense",
    "nf_moe_ep_transport", "nf_tp_split", "nf_tp_create", "nf_tp_destroy", "nf_tp_last_error", "nf_tp_transport",
    "nf_tp_linear_bf16", "nf_tp_argmax", "nf_tp_result", "nf_tp_sync", "nf_stack_create", "nf_stack_destroy",
    "nf_stack_last_error", "nf_stack_layer_ffn", "nf_stack_bind_bf16", "nf_stack_bind_f32", "nf_stack_finalize",
    "nf_stack_kv_cache", "nf_stack_decode", "nf_stack_sync", "nf_stack_load_kv", "nf_stack_fill_kv",
]
STAGES = ["router", "permute", "gate_up", "down", "shared", "combine"]


class Desc(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("inter", ctypes.c_int32), ("shared_inter", ctypes.c_int32), ("n_group", ctypes.c_int32),
        ("topk_group", ctypes.c_int32), ("normalize", ctypes.c_int32), ("routed_scaling", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float), ("expert_kind", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
    ]


class StackDesc(ctypes.Structure):
    _fields_ = [
        ("vocab", ctypes.c_int32), ("hidden", ctypes.c_int32), ("layers", ctypes.c_int32),
        ("dense_layers", ctypes.c_int32), ("bf16_expert_layers", ctypes.c_int32), ("dense_inter", ctypes.c_int32),
        ("moe", Desc), ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float), ("max_batch", ctypes.c_int32),
        ("max_context", ctypes.c_int32),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Loads the library (raises when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with python build.py")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I32, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    sig = {
        "nf_moe_create": ([ctypes.POINTER(Desc), I32, ctypes.POINTER(P)], I32),
        "nf_moe_destroy": ([P], None),
        "nf_moe_last_error": ([P], ctypes.c_char_p),
        "nf_status_string": ([I32], ctypes.c_char_p),
        "nf_moe_bind_nvfp4": ([P, I32, I32, P, P, F, F, I64, I64], I32),
        "nf_moe_bind_bf16": ([P, I32, I32, P, I64, I64], I32),
        "nf_moe_bind_f32": ([P, I32, P, I64], I32),
        "nf_moe_finalize": ([P], I32),
        "nf_moe_forward": ([P, P, P, I32, P, P, P, P], I32),
        "nf_moe_forward_host": ([P, P, P, I32, P, P, P], I32),
        "nf_moe_sync": ([P, P], I32),
        "nf_moe_route": ([P, P, I32, P, P, P, P], I32),
        "nf_moe_debug_tensor": ([P, I32, ctypes.POINTER(P), ctypes.POINTER(I64)], I32),
        "nf_moe_debug_read": ([P, I32, P, I64], I32),
        "nf_nvfp4_dequantize": ([P, P, F, I64, I64, P, P], I32),
        "nf_nvfp4_quantize": ([P, I64, I64, F, P, P, P, P], I32),
        "nf_sigmoid_ref": ([P, I64, P, P], I32),
        "nf_moe_profile": ([P, I32], I32),
        "nf_moe_set_graph_mode": ([P, I32], I32),
        "nf_moe_set_expert_gemm": ([P, I32], I32),
        "nf_format_selfcheck": ([ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I64)], I32),
        "nf_moe_stage_times": ([P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(I32)], I32),
        "nf_router_topk_noalloc": ([P, P, P, I32, I32, I32, I32, I32, I32, I32, F, P, P, ctypes.c_char_p, I32, P],
                                   I32),
        "nf_ep_unique_id": ([ctypes.c_char_p, I32], I32),
        "nf_moe_create_ep": ([ctypes.POINTER(Desc), I32, I32, I32, ctypes.c_char_p, I32, ctypes.POINTER(P)], I32),
        "nf_moe_create_ep_replicated": ([ctypes.POINTER(Desc), I32, I32, I32, ctypes.c_char_p, I32,
                                         ctypes.POINTER(ctypes.c_int32), I32, ctypes.POINTER(P)], I32),
        "nf_moe_create_dense": ([I32, I32, F, I32, I32, ctypes.POINTER(P)], I32),
        "nf_moe_ep_transport": ([P], I32),
        "nf_tp_split": ([I64, I32, I32, ctypes.POINTER(I64), ctypes.POINTER(I64)], I32),
        "nf_tp_create": ([I32, I32, I32, ctypes.c_char_p, I32, I32, I64, ctypes.POINTER(P)], I32),
        "nf_tp_destroy": ([P], None),
        "nf_tp_last_error": ([P], ctypes.c_char_p),
        "nf_tp_transport": ([P], I32),
        "nf_tp_linear_bf16": ([P, P, I64, I64, P, I32, P, P], I32),
        "nf_tp_argmax": ([P, I32, I64, P, P], I32),
        "nf_tp_result": ([P, ctypes.POINTER(P)], I32),
        "nf_tp_sync": ([P, P], I32),
        "nf_stack_create": ([ctypes.POINTER(StackDesc), I32, ctypes.POINTER(P)], I32),
        "nf_stack_destroy": ([P], None),
        "nf_stack_last_error": ([P], ctypes.c_char_p),
        "nf_stack_layer_ffn": ([P, I32], P),
        "nf_stack_bind_bf16": ([P, I32, I32, P, I64, I64], I32),
        "nf_stack_bind_f32": ([P, I32, I32, P, I64], I32),
        "nf_stack_finalize": ([P], I32),
        "nf_stack_kv_cache": ([P, I32, ctypes.POINTER(P), ctypes.POINTER(P)], I32),
        "nf_stack_decode": ([P, P, P, I32, P, P, P], I32),
        "nf_stack_sync": ([P, P], I32),
        "nf_stack_load_kv": ([P, I32, P, P], I32),
        "nf_stack_fill_kv": ([P, ctypes.c_uint64], I32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"]
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


class NfError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{NF_ERR.get(status, status)}]")
        self.status = status


_X_DTYPES = ("torch.int16", "torch.uint16", "torch.bfloat16")


def _dev(a, need: int, dtypes: tuple, name: str, device: int) -> int | None:
    """The device pointer of a buffer the library reads or writes `need`
    elements of.  A torch tensor must be a contiguous CUDA tensor on the
    handle's device with one of `dtypes` and at least `need` elements; a host
    array is refused (the kernels would fault on it).  A raw integer pointer is
    the caller's responsibility, as in the C ABI."""
    if a is None or isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        raise NfError(1, f"{name} is a host array; the device-buffer calls take CUDA tensors or device pointers")
    if not getattr(a, "is_cuda", False) or a.device.index != device:
        raise NfError(1, f"{name} is not on cuda:{device}" if device >= 0 else f"{name} is not a CUDA tensor")
    if str(a.dtype) not in dtypes:
        raise NfError(1, f"{name} has dtype {a.dtype}; expected {' or '.join(d[6:] for d in dtypes)}")
    if not a.is_contiguous():
        raise NfError(1, f"{name} is not contiguous")
    if a.numel() < need:
        raise NfError(1, f"{name} holds {a.numel()} elements; {need} needed")
    return a.data_ptr()


class MoeLayer:
    """One MoE layer resident on one GPU."""

    def __init__(self, hidden: int, experts: int, top_k: int, inter: int, shared_inter: int, *,
                 routed_scaling: float = 1.0, swiglu_limit: float = 10.0, n_group: int = 1, topk_group: int = 1,
                 normalize: bool = True, bf16_experts: bool = False, max_tokens: int = 64, device: int = 0,
                 ep: tuple[int, int, bytes] | None = None, ep_replicas=None):
        """ep = (rank, world, group_id) makes this rank's handle of an expert-
        parallel group (group_id from ep_group_id() on one rank, shared by all);
        max_tokens is then per rank.  ep_replicas: expert ids every rank also
        holds (the same list on every rank); picks of them stay on the rank of
        their token (nf_moe_create_ep_replicated)."""
        self.lib = load()
        self.desc = Desc(hidden, experts, top_k, inter, shared_inter, n_group, topk_group, int(normalize),
                         routed_scaling, swiglu_limit, EXPERTS_BF16 if bf16_experts else EXPERTS_NVFP4, max_tokens)
        h = ctypes.c_void_p()
        if ep is None:
            st = self.lib.nf_moe_create(ctypes.byref(self.desc), device, ctypes.byref(h))
        else:
            rank, world, group_id = ep
            if ep_replicas:
                reps = (ctypes.c_int32 * len(ep_replicas))(*[int(e) for e in ep_replicas])
                st = self.lib.nf_moe_create_ep_replicated(ctypes.byref(self.desc), device, rank, world, group_id,
                                                          len(group_id), reps, len(ep_replicas), ctypes.byref(h))
            else:
                st = self.lib.nf_moe_create_ep(ctypes.byref(self.desc), device, rank, world, group_id, len(group_id),
                                               ctypes.byref(h))
        if st != NF_OK:
            raise NfError(st, self.lib.nf_moe_last_error(None).decode())
        self.h = h
        self.device = device
        self.ep = ep

    @classmethod
    def borrow(cls, handle: int, desc: Desc, device: int) -> "MoeLayer":
        """A view of a handle another object owns (a decoder stack's layer):
        binding and forwards work, close() leaves the handle alone."""
        self = cls.__new__(cls)
        self.lib, self.desc, self.h, self.device, self.ep = load(), desc, ctypes.c_void_p(handle), device, None
        self.borrowed = True
        return self

    def close(self) -> None:
        if getattr(self, "borrowed", False):
            self.h = None
            return
        if getattr(self, "h", None):
            self.lib.nf_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int) -> None:
        if st != NF_OK:
            raise NfError(st, self.lib.nf_moe_last_error(self.h).decode())

    # ---- binding -----------------------------------------------------------
    def _proj_label(self, expert: int, proj: int) -> str:
        """The tensor prefix the library's messages name (proj_label in
        csrc/nf_moe.cu)."""
        return f"mlp.experts.{expert}.{_PROJ_NAMES.get(proj, 'proj')}"

    def bind_nvfp4(self, expert: int, proj: int, packed: np.ndarray, scales: np.ndarray, weight_scale_2: float,
                   input_scale: float) -> None:
        """Codes U8 [rows, cols / 2] and E4M3 block scales [rows, cols / 16].
        The arrays' ranks and the scales' shape are checked here as
        linear_nvfp4 checks them (src/text_forward.cpp:837-843): the C ABI takes
        only rows and cols, so a shorter scale array would be read past its end."""
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.uint8)
        if packed.ndim != 2 or scales.ndim != 2:
            raise NfError(3, f"NVFP4 layout {self._proj_label(expert, proj)}")
        rows, half = packed.shape
        if scales.shape != (rows, 2 * half // 16):
            raise NfError(2, f"NVFP4 shape {self._proj_label(expert, proj)}")
        self._check(self.lib.nf_moe_bind_nvfp4(self.h, expert, proj, _ptr(packed), _ptr(scales),
                                               float(weight_scale_2), float(input_scale), rows, 2 * half))

    def bind_bf16(self, which: int, data: np.ndarray, expert: int = 0) -> None:
        data = np.ascontiguousarray(data, dtype=np.uint16)
        rows, cols = data.shape
        self._check(self.lib.nf_moe_bind_bf16(self.h, which, expert, _ptr(data), rows, cols))

    def bind_f32(self, which: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data, dtype=np.float32)
        self._check(self.lib.nf_moe_bind_f32(self.h, which, _ptr(data), data.size))

    def finalize(self) -> None:
        self._check(self.lib.nf_moe_finalize(self.h))

    def bind_layer(self, lay) -> None:
        """Binds a workload.Layer and finalizes."""
        self.bind_bf16(BF16_ROUTER, lay.router_w)
        self.bind_f32(F32_ROUTER_BIAS, lay.bias)
        if lay.shared_inter > 0:
            self.bind_bf16(BF16_SHARED_GATE, lay.shared_gate)
            self.bind_bf16(BF16_SHARED_UP, lay.shared_up)
            self.bind_bf16(BF16_SHARED_DOWN, lay.shared_down)
        for e in range(lay.experts):
            if lay.bf16_experts:
                self.bind_bf16(BF16_EXPERT_GATE, lay.gate_bf16[e], e)
                self.bind_bf16(BF16_EXPERT_UP, lay.up_bf16[e], e)
                self.bind_bf16(BF16_EXPERT_DOWN, lay.down_bf16[e], e)
            else:
                self.bind_nvfp4(e, PROJ_GATE, lay.gate_packed[e], lay.gate_scales[e], lay.gate_ws2[e], lay.gate_in[e])
                self.bind_nvfp4(e, PROJ_UP, lay.up_packed[e], lay.up_scales[e], lay.up_ws2[e], lay.up_in[e])
                self.bind_nvfp4(e, PROJ_DOWN, lay.down_packed[e], lay.down_scales[e], lay.down_ws2[e], lay.down_in[e])
        self.finalize()

    def bind_from_store(self, store: Mapping[str, np.ndarray], prefix: str) -> None:
        """Binds every tensor of one MoE layer by checkpoint name, e.g.
        prefix = "model.language_model.layers.3." (names as in
        parameter_schema add_moe, src/parameter_schema.cpp:72-98).  A missing
        name raises "missing tensor <name>" like Store::get
        (src/text_forward.cpp:462-466)."""

        def get(name: str) -> np.ndarray:
            if name not in store:
                raise NfError(5, f"missing tensor {name}")
            return np.asarray(store[name])

        self.bind_bf16(BF16_ROUTER, get(prefix + "mlp.gate.weight"))
        self.bind_f32(F32_ROUTER_BIAS, get(prefix + "mlp.gate.e_score_correction_bias"))
        if self.desc.shared_inter > 0:
            self.bind_bf16(BF16_SHARED_GATE, get(prefix + "mlp.shared_experts.gate_proj.weight"))
            self.bind_bf16(BF16_SHARED_UP, get(prefix + "mlp.shared_experts.up_proj.weight"))
            self.bind_bf16(BF16_SHARED_DOWN, get(prefix + "mlp.shared_experts.down_proj.weight"))
        for e in range(self.desc.experts):
            base = f"{prefix}mlp.experts.{e}."
            for proj, name in ((PROJ_GATE, "gate_proj"), (PROJ_UP, "up_proj"), (PROJ_DOWN, "down_proj")):
                if self.desc.expert_kind == EXPERTS_BF16:
                    self.bind_bf16(BF16_EXPERT_GATE + proj, get(base + name + ".weight"), e)
                else:
                    self._bind_nvfp4_named(get, base + name, e, proj)
        self.finalize()

    def _bind_nvfp4_named(self, get, name: str, expert: int, proj: int) -> None:
        """One NVFP4 linear by checkpoint name: <name>.weight, .weight_scale and
        the rank-0 F32 .weight_scale_2 / .input_scale (linear_nvfp4's lookups,
        src/text_forward.cpp:833-836)."""
        ws2 = get(name + ".weight_scale_2")
        ins = get(name + ".input_scale")
        if ws2.ndim != 0 or ins.ndim != 0:
            raise NfError(3, f"expected rank-0 F32 for {name}.weight_scale_2")
        self.bind_nvfp4(expert, proj, get(name + ".weight"), get(name + ".weight_scale"), float(ws2), float(ins))

    # ---- execution ---------------------------------------------------------
    def forward(self, x_dev, y_dev, tokens: int, residual_dev=None, idx_dev=None, w_dev=None, stream=0) -> None:
        """Device-buffer forward (asynchronous on `stream`).  Tensors are checked
        for device, dtype, contiguity and size before the call (x BF16 bits
        [tokens, H]; residual and y fp32 [tokens, H]; idx int32 and w fp32
        [tokens, k]); a token count outside 0..max_tokens is the library's to
        reject."""
        H, K, d = self.desc.hidden, self.desc.top_k, self.device
        n = tokens if 0 <= tokens <= self.desc.max_tokens else 0
        f32, i32 = ("torch.float32",), ("torch.int32",)
        self._check(self.lib.nf_moe_forward(self.h, _dev(x_dev, n * H, _X_DTYPES, "x", d),
                                            _dev(residual_dev, n * H, f32, "residual", d), tokens,
                                            _dev(y_dev, n * H, f32, "y", d), _dev(idx_dev, n * K, i32, "idx", d),
                                            _dev(w_dev, n * K, f32, "w", d), stream or None))

    def forward_host(self, x: np.ndarray, residual: np.ndarray | None = None, with_routes: bool = False,
                     out: tuple | None = None):
        """Host fp32 in / fp32 out, the reference's own moe() contract.  out =
        (y, idx, w) reuses caller-owned host arrays (page-locked ones make the
        device-to-host copies direct); idx and w may be None."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        H = self.desc.hidden
        # the library copies tokens x hidden floats from each host array
        if x.ndim != 2 or x.shape[1] != H:
            raise ValueError(f"x must be [tokens, {H}] float32")
        T = x.shape[0]
        if residual is not None and np.shape(residual) != x.shape:
            raise ValueError("residual must have x's shape")
        if out is not None:
            y, idx, w = out
            for a, shape, dt in ((y, x.shape, np.float32), (idx, (T, self.desc.top_k), np.int32),
                                 (w, (T, self.desc.top_k), np.float32)):
                if a is not None and (a.shape != shape or a.dtype != dt or not a.flags["C_CONTIGUOUS"]):
                    raise ValueError("out arrays must be contiguous with the forward's shapes and dtypes")
            with_routes = idx is not None or w is not None
        else:
            y = np.empty_like(x)
            idx = np.empty((T, self.desc.top_k), np.int32) if with_routes else None
            w = np.empty((T, self.desc.top_k), np.float32) if with_routes else None
        res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        self._check(self.lib.nf_moe_forward_host(self.h, _ptr(x), _ptr(res), T, _ptr(y), _ptr(idx), _ptr(w)))
        return (y, idx, w) if with_routes else y

    def route(self, x_dev, tokens: int, logits_dev=None, idx_dev=None, w_dev=None, stream=0) -> None:
        """The router alone: logits fp32 [tokens, E], idx int32 and w fp32
        [tokens, k] (each optional), checked as in forward."""
        H, E, K, d = self.desc.hidden, self.desc.experts, self.desc.top_k, self.device
        n = tokens if 0 <= tokens <= self.desc.max_tokens else 0
        f32, i32 = ("torch.float32",), ("torch.int32",)
        self._check(self.lib.nf_moe_route(self.h, _dev(x_dev, n * H, _X_DTYPES, "x", d), tokens,
                                          _dev(logits_dev, n * E, f32, "logits", d),
                                          _dev(idx_dev, n * K, i32, "idx", d), _dev(w_dev, n * K, f32, "w", d),
                                          stream or None))

    def ep_transport(self) -> str:
        """"none" (one GPU), "nccl" or "nvlink" (the EP exchange in use)."""
        return {0: "none", 1: "nccl", 2: "nvlink"}[self.lib.nf_moe_ep_transport(self.h)]

    def sync(self, stream=0) -> None:
        self._check(self.lib.nf_moe_sync(self.h, stream or None))

    def debug_tensor(self, which: str) -> tuple[int, int]:
        p = ctypes.c_void_p()
        n = ctypes.c_int64()
        self._check(self.lib.nf_moe_debug_tensor(self.h, DBG[which], ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def set_graph_mode(self, enable: bool) -> None:
        """Capture forwards into CUDA graphs and replay them (needs a stream)."""
        self._check(self.lib.nf_moe_set_graph_mode(self.h, int(enable)))

    def set_expert_gemm(self, mode: str) -> None:
        """The prefill-size expert GEMM form: "one_sm" (default), "wide" or "pair"."""
        self._check(self.lib.nf_moe_set_expert_gemm(self.h, EXPERT_GEMM[mode]))

    def profile(self, enable: bool) -> None:
        """Start (and clear) or stop per-stage CUDA-event timing."""
        self._check(self.lib.nf_moe_profile(self.h, int(enable)))

    def stage_times(self) -> tuple[dict, int]:
        """Accumulated device milliseconds per stage and the forwards counted."""
        ms = (ctypes.c_float * len(STAGES))()
        n = ctypes.c_int()
        self._check(self.lib.nf_moe_stage_times(self.h, ms, ctypes.byref(n)))
        return {name: float(ms[i]) for i, name in enumerate(STAGES)}, n.value

    def debug_read(self, which: str, dtype, count: int) -> np.ndarray:
        """Host copy of the first `count` elements of an internal buffer."""
        out = np.empty(count, dtype)
        self._check(self.lib.nf_moe_debug_read(self.h, DBG[which], _ptr(out), out.nbytes))
        return out


class DenseMlp(MoeLayer):
    """The dense NVFP4 MLP of the first layers (TextModel::dense_mlp,
    src/text_forward.cpp:909-915) resident on one GPU: a one-expert handle
    without a router (nf_moe_create_dense) whose gate/up epilogue applies
    swiglu_clamp_bf16.  forward() / forward_host() take no route buffers."""

    def _proj_label(self, expert: int, proj: int) -> str:
        return f"mlp.{_PROJ_NAMES.get(proj, 'proj')}"

    def __init__(self, hidden: int, inter: int, *, swiglu_limit: float = 10.0, max_tokens: int = 64,
                 device: int = 0):
        self.lib = load()
        h = ctypes.c_void_p()
        st = self.lib.nf_moe_create_dense(hidden, inter, swiglu_limit, max_tokens, device, ctypes.byref(h))
        if st != NF_OK:
            raise NfError(st, self.lib.nf_moe_last_error(None).decode())
        self.desc = Desc(hidden, 1, 1, inter, 0, 1, 1, 1, 1.0, swiglu_limit, EXPERTS_NVFP4, max_tokens)
        self.h = h
        self.device = device
        self.ep = None

    def bind_layer(self, lay) -> None:
        """Binds a workload.DenseLayer and finalizes."""
        self.bind_nvfp4(0, PROJ_GATE, lay.gate_packed, lay.gate_scales, lay.gate_ws2, lay.gate_in)
        self.bind_nvfp4(0, PROJ_UP, lay.up_packed, lay.up_scales, lay.up_ws2, lay.up_in)
        self.bind_nvfp4(0, PROJ_DOWN, lay.down_packed, lay.down_scales, lay.down_ws2, lay.down_in)
        self.finalize()

    def bind_from_store(self, store: Mapping[str, np.ndarray], prefix: str) -> None:
        """Binds <prefix>mlp.{gate,up,down}_proj by checkpoint name (the dense
        layers' names, src/parameter_schema.cpp:187-191) and finalizes."""

        def get(name: str) -> np.ndarray:
            if name not in store:
                raise NfError(5, f"missing tensor {name}")
            return np.asarray(store[name])

        for proj, name in ((PROJ_GATE, "gate_proj"), (PROJ_UP, "up_proj"), (PROJ_DOWN, "down_proj")):
            self._bind_nvfp4_named(get, f"{prefix}mlp.{name}", 0, proj)
        self.finalize()

    def forward(self, x_dev, y_dev, tokens: int, residual_dev=None, idx_dev=None, w_dev=None, stream=0) -> None:
        if idx_dev is not None or w_dev is not None:
            raise NfError(1, "a dense MLP has no routes")
        super().forward(x_dev, y_dev, tokens, residual_dev, None, None, stream)


_ST_DTYPES = {"BF16": np.uint16, "F32": np.float32, "U8": np.uint8, "F8_E4M3": np.uint8}


def safetensors_store(directory) -> dict:
    """Name -> read-only memory-mapped array over a safetensors checkpoint
    directory (model.safetensors.index.json and its shards, or a single
    model.safetensors), for MoeLayer / DenseMlp.bind_from_store.  The Python
    twin of host/nf_safetensors.hpp, with the reference Store's messages
    (src/text_forward.cpp:328-495) and the same range and size checks."""
    import json
    from pathlib import Path

    d = Path(directory)
    index = d / "model.safetensors.index.json"
    if index.is_file():
        text = index.read_text()
        if not text:
            raise NfError(3, "empty safetensors index")
        wmap = json.loads(text).get("weight_map")
        if wmap is None:
            raise NfError(3, "index has no weight_map")
        shards = list(dict.fromkeys(wmap.values()))
    elif (d / "model.safetensors").is_file():
        shards = ["model.safetensors"]
    else:
        raise NfError(3, "missing model.safetensors.index.json")
    out = {}
    for shard in shards:
        path = d / shard
        if not path.is_file():
            raise NfError(3, f"cannot open shard {path}")
        raw = np.memmap(path, dtype=np.uint8, mode="r")
        if raw.size < 8:
            raise NfError(3, "short safetensors file")
        hlen = int(raw[:8].view("<u8")[0])
        if hlen == 0 or hlen > raw.size - 8:
            raise NfError(3, "bad safetensors header")
        try:
            header = json.loads(bytes(raw[8:8 + hlen]).decode())
        except ValueError:
            raise NfError(3, "bad safetensors header") from None
        data = raw[8 + hlen:]
        for name, info in header.items():
            if name == "__metadata__":
                continue
            dt = _ST_DTYPES.get(info.get("dtype"))
            if dt is None:
                raise NfError(3, f"unsupported dtype {info.get('dtype')} for {name}")
            shape, offs = info.get("shape"), info.get("data_offsets")
            if shape is None or offs is None:
                raise NfError(3, f"incomplete tensor header for {name}")
            if len(shape) > 8:
                raise NfError(3, f"rank above 8 for {name}")
            shape = [int(v) for v in shape]
            if any(v < 0 for v in shape):
                raise NfError(3, f"negative dimension for {name}")
            b, e = int(offs[0]), int(offs[1])
            if b < 0 or e < b or e > data.size:
                raise NfError(3, f"tensor data out of range for {name}")
            # (Python integers: the element count cannot wrap)
            if math.prod(shape) * np.dtype(dt).itemsize != e - b:
                raise NfError(3, f"tensor size mismatch for {name}")
            out[name] = data[b:e].view(dt).reshape(shape)
    return out


_U8, _F32 = ("torch.uint8",), ("torch.float32",)


def _dev_all(specs) -> tuple:
    """_dev over (buffer, elements, dtypes, name) specs on the current device
    (the one these free functions run on)."""
    d = _current_device() if any(getattr(a, "is_cuda", False) for a, *_ in specs) else -1
    return tuple(_dev(a, max(int(n), 0), dt, name, d) for a, n, dt, name in specs)


# The format helpers below return the library's status like the C ABI; a
# buffer refused on the host (a host array, another device, a dtype or size
# the call cannot use) returns NF_ERR_INVALID without calling the library.
def dequantize(packed_dev, scales_dev, global_scale: float, rows: int, cols: int, out_dev, stream=0) -> int:
    """packed U8 [rows, cols / 2], scales U8 [rows, cols / 16] -> out F32
    [rows, cols] (device buffers)."""
    try:
        p = _dev_all(((packed_dev, rows * cols // 2, _U8, "packed"), (scales_dev, rows * cols // 16, _U8, "scales"),
                      (out_dev, rows * cols, _F32, "out")))
    except NfError as e:
        return e.status
    return load().nf_nvfp4_dequantize(p[0], p[1], global_scale, rows, cols, p[2], stream or None)


def quantize(x_dev, rows: int, cols: int, input_scale: float, codes_dev, scales_dev, fake_dev=None, stream=0) -> int:
    """x F32 [rows, cols] -> codes U8 [rows, cols / 2], scales U8 [rows,
    cols / 16], optional fake-quant F32 [rows, cols] (device buffers)."""
    try:
        p = _dev_all(((x_dev, rows * cols, _F32, "x"), (codes_dev, rows * cols // 2, _U8, "codes"),
                      (scales_dev, rows * cols // 16, _U8, "scales"), (fake_dev, rows * cols, _F32, "fake")))
    except NfError as e:
        return e.status
    return load().nf_nvfp4_quantize(p[0], rows, cols, input_scale, p[1], p[2], p[3], stream or None)


def sigmoid_ref(x_dev, n: int, y_dev, stream=0) -> int:
    """y = sigmoid(x) over n F32 elements (device buffers)."""
    try:
        p = _dev_all(((x_dev, n, _F32, "x"), (y_dev, n, _F32, "y")))
    except NfError as e:
        return e.status
    return load().nf_sigmoid_ref(p[0], n, p[1], stream or None)


NOALLOC_MAX_SCORES = 16384  # tokens x experts of one nf_router_topk_noalloc call


def _current_device() -> int:
    """The CUDA device the library's calls run on (torch's current device)."""
    import torch

    return torch.cuda.current_device() if torch.cuda.is_available() else 0


def router_topk_noalloc(x_dev, router_w_dev, bias_dev, tokens: int, hidden: int, experts: int, top_k: int,
                        idx_dev, w_dev, *, n_group: int = 1, topk_group: int = 1, normalize: bool = True,
                        routed_scaling: float = 1.0, stream=0) -> tuple[int, str]:
    """Router top-k from caller device buffers with no device allocation
    (the library's static scratch; calls must not overlap).  Returns
    (status, message).

    Every tensor is checked before the library is called, as in
    MoeLayer.forward: a CUDA tensor on the current device (the scratch and
    the launches use that device), contiguous, with the documented dtype and
    at least the elements the call reads or writes (x BF16 bits [tokens,
    hidden], router weights BF16 bits [experts, hidden], bias fp32 [experts],
    idx int32 and w fp32 [tokens, top_k]).  A host array raises NfError: the
    router's bulk copies would read it as a device address."""
    d = -1
    if any(getattr(a, "is_cuda", False) for a in (x_dev, router_w_dev, bias_dev, idx_dev, w_dev)):
        d = _current_device()
    n = tokens if tokens >= 0 else 0
    e = experts if experts >= 0 else 0
    f32, i32 = ("torch.float32",), ("torch.int32",)
    ptrs = (_dev(x_dev, n * max(hidden, 0), _X_DTYPES, "x", d),
            _dev(router_w_dev, e * max(hidden, 0), _X_DTYPES, "router_w", d),
            _dev(bias_dev, e, f32, "bias", d),
            _dev(idx_dev, n * max(top_k, 0), i32, "idx", d),
            _dev(w_dev, n * max(top_k, 0), f32, "w", d))
    buf = ctypes.create_string_buffer(256)
    st = load().nf_router_topk_noalloc(ptrs[0], ptrs[1], ptrs[2], tokens, hidden, experts, top_k, n_group, topk_group,
                                       int(normalize), routed_scaling, ptrs[3], ptrs[4], buf, len(buf), stream or None)
    return st, buf.value.decode()


EP_ID_BYTES = 128


def tp_split(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Row block [row0, row1) that rank `rank` of `world` computes."""
    a, b = ctypes.c_int64(), ctypes.c_int64()
    st = load().nf_tp_split(rows, rank, world, ctypes.byref(a), ctypes.byref(b))
    if st != NF_OK:
        raise NfError(st, "bad tensor-parallel split arguments")
    return a.value, b.value


class TpGroup:
    """This rank's handle of a tensor-parallel group (nf_tp_*): BF16 linears
    split by output rows over `world` GPUs with the rows gathered on every
    rank, the GPU form of the reference's apply_rows + gather_rows
    (src/text_forward.cpp:242-256, 803-830).  group_id from ep_group_id() on
    one rank, shared by all (not needed for world = 1)."""

    def __init__(self, max_tokens: int, max_rows: int, *, rank: int = 0, world: int = 1,
                 group_id: bytes | None = None, device: int = 0):
        self.lib = load()
        h = ctypes.c_void_p()
        gid = group_id if group_id is not None else None
        st = self.lib.nf_tp_create(device, rank, world, gid, len(gid) if gid else 0, max_tokens, max_rows,
                                   ctypes.byref(h))
        if st != NF_OK:
            raise NfError(st, self.lib.nf_tp_last_error(None).decode())
        self.h, self.rank, self.world, self.device = h, rank, world, device
        self.max_tokens, self.max_rows = max_tokens, max_rows

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.nf_tp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int) -> None:
        if st != NF_OK:
            raise NfError(st, self.lib.nf_tp_last_error(self.h).decode())

    def split(self, rows: int) -> tuple[int, int]:
        return tp_split(rows, self.rank, self.world)

    def transport(self) -> str:
        return {0: "none", 1: "nccl", 2: "nvlink"}[self.lib.nf_tp_transport(self.h)]

    def linear_bf16(self, w_shard, rows: int, cols: int, x, tokens: int, y=None, stream=0) -> None:
        """linear_bf16 on this rank's rows: w_shard BF16 bits [row1 - row0, cols]
        (see split), x fp32 [tokens, cols]; y fp32 [tokens, rows] (optional)
        receives the whole output.  Checked like MoeLayer.forward."""
        r0, r1 = self.split(rows)
        d = self.device
        n = tokens if 0 <= tokens <= self.max_tokens else 0
        self._check(self.lib.nf_tp_linear_bf16(self.h, _dev(w_shard, (r1 - r0) * cols, _X_DTYPES, "w_shard", d),
                                               rows, cols, _dev(x, n * cols, ("torch.float32",), "x", d), tokens,
                                               _dev(y, n * rows, ("torch.float32",), "y", d), stream or None))

    def argmax(self, tokens: int, rows: int, idx, stream=0) -> None:
        """The reference's greedy pick over the last linear's output: idx int32 [tokens]."""
        n = tokens if 0 <= tokens <= self.max_tokens else 0
        self._check(self.lib.nf_tp_argmax(self.h, tokens, rows, _dev(idx, n, ("torch.int32",), "idx", self.device),
                                          stream or None))

    def sync(self, stream=0) -> None:
        self._check(self.lib.nf_tp_sync(self.h, stream or None))


def ep_group_id() -> bytes:
    """A new expert-parallel group id (NCCL unique id) to hand to every rank."""
    buf = ctypes.create_string_buffer(EP_ID_BYTES)
    st = load().nf_ep_unique_id(buf, EP_ID_BYTES)
    if st != NF_OK:
        raise NfError(st, load().nf_moe_last_error(None).decode())
    return buf.raw


def format_selfcheck() -> tuple[int, int, int]:
    """(E2M1, E4M3, BF16) mismatch counts of the hardware conversions against
    the reference encoders over every 32-bit pattern (current device)."""
    a, b, c = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    st = load().nf_format_selfcheck(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    if st != NF_OK:
        raise NfError(st, "format self-check failed to run")
    return a.value, b.value, c.value


def sf_atom_offset(row: np.ndarray, kgroup: np.ndarray, kgroups_total: int) -> np.ndarray:
    """Byte offset of block scale (row, kgroup) in the tcgen05 atom layout."""
    row = np.asarray(row, dtype=np.int64)
    kgroup = np.asarray(kgroup, dtype=np.int64)
    atom = (row >> 7) * (kgroups_total >> 2) + (kgroup >> 2)
    return atom * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (kgroup & 3)


def sf_from_atoms(atoms: np.ndarray, rows: int, kgroups: int) -> np.ndarray:
    """Row-major [rows, kgroups] scales from the atom layout."""
    r = np.arange(rows)[:, None]
    k = np.arange(kgroups)[None, :]
    return np.asarray(atoms)[sf_atom_offset(r, k, kgroups)]


STACK_EMBED, STACK_LM_HEAD, STACK_Q_PROJ, STACK_K_PROJ, STACK_V_PROJ, STACK_O_PROJ = 0, 1, 2, 3, 4, 5
STACK_ATTN_NORM, STACK_FFN_NORM, STACK_Q_NORM, STACK_K_NORM, STACK_FINAL_NORM = 6, 7, 8, 9, 10


class DecoderStack:
    """A decoder stack for greedy decode on one GPU (nf_stack_*): embedding,
    per layer GQA attention + the layer's feed-forward (dense NVFP4 MLP,
    NVFP4 MoE, BF16-expert MoE), final norm, lm_head and greedy pick -- the
    reference's TextModel::step + argmax (src/text_forward.cpp:625-698)."""

    def __init__(self, *, vocab: int, hidden: int, layers: int, dense_layers: int, bf16_expert_layers: int,
                 dense_inter: int, experts: int, top_k: int, inter: int, shared_inter: int, routed_scaling: float,
                 swiglu_limit: float = 10.0, q_heads: int, kv_heads: int, head_dim: int = 128,
                 rope_theta: float = 10000.0, norm_eps: float = 1e-5, max_batch: int = 1, max_context: int = 2048,
                 device: int = 0):
        self.lib = load()
        moe = Desc(hidden, experts, top_k, inter, shared_inter, 1, 1, 1, routed_scaling, swiglu_limit, EXPERTS_NVFP4,
                   max_batch)
        self.desc = StackDesc(vocab, hidden, layers, dense_layers, bf16_expert_layers, dense_inter, moe, q_heads,
                              kv_heads, head_dim, rope_theta, norm_eps, max_batch, max_context)
        h = ctypes.c_void_p()
        st = self.lib.nf_stack_create(ctypes.byref(self.desc), device, ctypes.byref(h))
        if st != NF_OK:
            raise NfError(st, self.lib.nf_stack_last_error(None).decode())
        self.h, self.device = h, device

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.nf_stack_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int) -> None:
        if st != NF_OK:
            raise NfError(st, self.lib.nf_stack_last_error(self.h).decode())

    def ffn(self, layer: int):
        """The layer's feed-forward handle (a borrowed MoeLayer / DenseMlp view)."""
        d = self.desc
        ptr = self.lib.nf_stack_layer_ffn(self.h, layer)
        if not ptr:
            raise NfError(1, f"layer {layer} out of range")
        if layer < d.dense_layers:
            desc = Desc(d.hidden, 1, 1, d.dense_inter, 0, 1, 1, 1, 1.0, d.moe.swiglu_limit, EXPERTS_NVFP4, d.max_batch)
            return DenseMlp.borrow(ptr, desc, self.device)
        bf16 = layer >= d.layers - d.bf16_expert_layers
        m = d.moe
        desc = Desc(d.hidden, m.experts, m.top_k, m.inter, m.shared_inter, 1, 1, 1, m.routed_scaling, m.swiglu_limit,
                    EXPERTS_BF16 if bf16 else EXPERTS_NVFP4, d.max_batch)
        return MoeLayer.borrow(ptr, desc, self.device)

    def bind_bf16(self, which: int, data: np.ndarray, layer: int = 0) -> None:
        data = np.ascontiguousarray(data, dtype=np.uint16)
        rows, cols = data.shape
        self._check(self.lib.nf_stack_bind_bf16(self.h, which, layer, _ptr(data), rows, cols))

    def bind_f32(self, which: int, data: np.ndarray, layer: int = 0) -> None:
        data = np.ascontiguousarray(data, dtype=np.float32)
        self._check(self.lib.nf_stack_bind_f32(self.h, which, layer, _ptr(data), data.size))

    def bind_model(self, model) -> None:
        """Binds a workload.StackModel (every layer's attention, norms and FFN)
        and finalizes."""
        self.bind_bf16(STACK_EMBED, model.embed)
        self.bind_bf16(STACK_LM_HEAD, model.lm_head)
        self.bind_f32(STACK_FINAL_NORM, model.final_norm)
        for l, ly in enumerate(model.layers):
            self.bind_bf16(STACK_Q_PROJ, ly.wq, l)
            self.bind_bf16(STACK_K_PROJ, ly.wk, l)
            self.bind_bf16(STACK_V_PROJ, ly.wv, l)
            self.bind_bf16(STACK_O_PROJ, ly.wo, l)
            self.bind_f32(STACK_ATTN_NORM, ly.attn_norm, l)
            self.bind_f32(STACK_FFN_NORM, ly.ffn_norm, l)
            self.bind_f32(STACK_Q_NORM, ly.q_norm, l)
            self.bind_f32(STACK_K_NORM, ly.k_norm, l)
            self.ffn(l).bind_layer(ly.ffn)
        self._check(self.lib.nf_stack_finalize(self.h))

    def kv_cache(self, layer: int) -> tuple[int, int]:
        """Device addresses of the layer's K and V caches (BF16 [max_batch]
        [kv_heads][max_context][128])."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self.lib.nf_stack_kv_cache(self.h, layer, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def load_kv(self, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        """Host BF16 bits [max_batch, kv_heads, max_context, 128] into the layer's caches."""
        d = self.desc
        shape = (d.max_batch, d.kv_heads, d.max_context, d.head_dim)
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        if k.shape != shape or v.shape != shape:
            raise NfError(2, f"cache arrays must be {shape}")
        self._check(self.lib.nf_stack_load_kv(self.h, layer, _ptr(k), _ptr(v)))

    def fill_kv(self, seed: int) -> None:
        """Every layer's caches filled on the device with pseudo-random BF16 values."""
        self._check(self.lib.nf_stack_fill_kv(self.h, seed))

    def decode(self, tokens_dev, positions_dev, batch: int, next_dev, final_dev=None, stream=0) -> None:
        """One greedy step: int32 tokens / positions [batch] -> int32 next [batch]
        (final fp32 [batch, H] optional).  Asynchronous on `stream`."""
        d, dv = self.desc, self.device
        n = batch if 0 <= batch <= d.max_batch else 0
        i32 = ("torch.int32",)
        self._check(self.lib.nf_stack_decode(self.h, _dev(tokens_dev, n, i32, "tokens", dv),
                                             _dev(positions_dev, n, i32, "positions", dv), batch,
                                             _dev(next_dev, n, i32, "next", dv),
                                             _dev(final_dev, n * d.hidden, ("torch.float32",), "final", dv),
                                             stream or None))

    def sync(self, stream=0) -> None:
        self._check(self.lib.nf_stack_sync(self.h, stream or None))
