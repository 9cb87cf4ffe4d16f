"""CPU oracle of the decoder stack's greedy step (TEST INFRASTRUCTURE ONLY).

Composes the checker primitives of oracle.py (the C restatement pinned to the
reference: rmsnorm, gemv_bf16, the MoE layer, the dense MLP) with a numpy
restatement of the reference's GQA attention math, draft_attention
(src/text_forward.cpp:1216-1289), for one new token per sequence:

  per head: q, k = rmsnorm(q / k; q_norm / k_norm, 1e-5)       (:1246-1257)
            q, k rotated by rope_heads at the token's position  (:1169-1184)
            score_j = (q . k_j) * 1/sqrt(128); weights = exp(score - max)
            mixed = sum_j (weight_j / sum) v_j                  (:1259-1286)
  o = gemv_bf16(o_proj, mixed)                                  (:1287)

The layer structure (pre-norm attention, rmsnorm_stash into the FFN, the
residual adds) is the stack's own, as nf_stack.cu documents it.  Only
tests/ use this module.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np


def _checker():
    """oracle.py (the ctypes access to the C checkers), loaded once."""
    name = "nf_oracle_py"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, Path(__file__).resolve().with_name("oracle.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


orc = _checker()

D = 128


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_f32(x: np.ndarray) -> np.ndarray:
    """x rounded to BF16 (round to nearest even), as F32 values."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)) << np.uint32(16)
    return r.view(np.float32)


def rmsnorm_rows(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """The reference's rmsnorm (sequential sum of squares) on every row."""
    lib = orc.port()
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.zeros_like(x)
    for r in range(x.shape[0]):
        lib.or_rmsnorm(orc.p(x[r]), orc.p(w), np.float32(eps), x.shape[1], orc.p(y[r]))
    return y


def rmsnorm_stash_rows(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rmsnorm_stash (src/text_forward.cpp:267-276): the sum of squares of x,
    then bf16(bf16(x) * inv * w)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[1]
    sq = np.zeros(x.shape[0], np.float32)
    for i in range(n):
        sq = (sq + x[:, i] * x[:, i]).astype(np.float32)
    inv = (np.float32(1) / np.sqrt((sq / np.float32(n) + np.float32(eps)).astype(np.float32))).astype(np.float32)
    return f32_to_bf16_f32((f32_to_bf16_f32(x) * inv[:, None]).astype(np.float32) * w[None, :])


def gemv_rows(w_bits: np.ndarray, x: np.ndarray) -> np.ndarray:
    """gemv_bf16 of every row of x: [T, rows]."""
    lib = orc.port()
    rows, cols = w_bits.shape
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    out = np.zeros((x.shape[0], rows), np.float32)
    for t in range(x.shape[0]):
        xt = np.ascontiguousarray(x[t], dtype=np.float32)
        lib.or_gemv_bf16(orc.p(w), orc.p(xt), rows, cols, 0, rows, orc.p(out[t]))
    return out


def rope(v: np.ndarray, position: int, theta: float = 10000.0) -> np.ndarray:
    """rope_heads on one head (src/text_forward.cpp:1169-1184), float math."""
    v = v.astype(np.float32).copy()
    i = np.arange(D // 2, dtype=np.float32)
    freq = np.power(np.float32(theta), (np.float32(-2.0) * i / np.float32(D)).astype(np.float32)).astype(np.float32)
    ang = (np.float32(position) * freq).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    first, second = v[: D // 2].copy(), v[D // 2:].copy()
    v[: D // 2] = first * c - second * s
    v[D // 2:] = first * s + second * c
    return v


def head_norm(v: np.ndarray, w: np.ndarray) -> np.ndarray:
    return rmsnorm_rows(v[None, :], w, 1e-5)[0]


def attention_token(q_heads: np.ndarray, keys: np.ndarray, values: np.ndarray) -> np.ndarray:
    """draft_attention's softmax-weighted sum for one token: q_heads [nq, D],
    keys / values [nkv, len, D] (F32) -> mixed [nq, D]."""
    nq, nkv = q_heads.shape[0], keys.shape[0]
    group = nq // nkv
    scale = np.float32(1.0) / np.sqrt(np.float32(D))
    out = np.zeros((nq, D), np.float32)
    for h in range(nq):
        g = h // group
        scores = (keys[g] @ q_heads[h]).astype(np.float32) * scale
        w = np.exp((scores - scores.max()).astype(np.float32)).astype(np.float32)
        out[h] = ((w / w.sum()).astype(np.float32)[:, None] * values[g]).sum(axis=0)
    return out


def decode_step(model, k_hist: list, v_hist: list, tokens: np.ndarray, positions: np.ndarray, eps: float = 1e-5):
    """One greedy step of the stack for every sequence.  k_hist[l] / v_hist[l]
    are the layers' caches as F32 [batch, nkv, L, D] holding positions
    < positions[i]; the new keys and values are written at positions[i]
    (rounded to BF16, as the stack stores them).  Returns (next tokens,
    logits [batch, vocab], final norm output [batch, H])."""
    cfg = model.cfg
    nq, nkv = cfg["q_heads"], cfg["kv_heads"]
    x = bf16_bits_to_f32(model.embed[tokens])
    for l, ly in enumerate(model.layers):
        a = rmsnorm_rows(x, ly.attn_norm, eps)
        q = gemv_rows(ly.wq, a).reshape(-1, nq, D)
        k = gemv_rows(ly.wk, a).reshape(-1, nkv, D)
        v = gemv_rows(ly.wv, a).reshape(-1, nkv, D)
        mixed = np.zeros((x.shape[0], nq * D), np.float32)
        for i, p in enumerate(positions):
            qh = np.stack([rope(head_norm(q[i, h], ly.q_norm), p) for h in range(nq)])
            for g in range(nkv):
                k_hist[l][i, g, p] = f32_to_bf16_f32(rope(head_norm(k[i, g], ly.k_norm), p))
                v_hist[l][i, g, p] = f32_to_bf16_f32(v[i, g])
            mixed[i] = attention_token(qh, k_hist[l][i, :, : p + 1], v_hist[l][i, :, : p + 1]).ravel()
        o = gemv_rows(ly.wo, mixed)
        h = (x + o).astype(np.float32)
        f = rmsnorm_stash_rows(h, ly.ffn_norm, eps)
        if hasattr(ly.ffn, "experts"):
            x = orc.moe_layer(orc.port(), ly.ffn, f, h)[0]
        else:
            x = orc.dense_mlp(orc.port(), ly.ffn, f, h)
    fin = rmsnorm_rows(x, model.final_norm, eps)
    logits = gemv_rows(model.lm_head, fin)
    nxt = np.zeros(len(tokens), np.int32)
    for i, row in enumerate(logits):
        if np.isnan(row[0]):
            continue
        ok = ~np.isnan(row)
        nxt[i] = int(np.nonzero(ok & (row == row[ok].max()))[0][0])
    return nxt, logits, fin
