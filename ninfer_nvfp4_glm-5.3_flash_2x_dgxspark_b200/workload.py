"""Seeded synthetic MoE-layer inputs with the shapes and value distributions of
the benchmark configurations (no checkpoint or dataset is involved):

  x            BF16 = RNE(N(0, 1))                         [T, H]
  router W     BF16 = RNE(N(0, 0.02))                      [E, H]
  bias         F32  ~ U(-0.1, 0.1)                         [E]
  NVFP4 codes  uniform over the 16 E2M1 nibbles            packed U8 [N, K/2]
  block scales E4M3(clamp(|N(0, 1)|, 2^-6, 448))           [N, K/16]
  weight_scale_2 = 1/448, input_scale = 1/6                per projection
  shared / BF16 experts BF16 = RNE(N(0, 0.02))

Configurations (the benchmark's configs list):
  c0 tiny     H256  E8  k2 I128  Is128 T16    scale 1.0
  c1 decode   H2048 E64 k4 I1536 Is1536 T64   scale 2.5
  c2 prefill  c1 with T8192 and the bias tuned so every expert gets 512 +- 10%
  c3 EP       c1 with T16384 and a Zipf(1.1) log-prior added to the bias, at
              the configuration's literal weight lambda = 1 and at a
              calibrated lambda (C3_LAMBDA_CALIBRATED)
  c4 dense    configs[4]'s dense NVFP4 MLP (layers 0-2): H2048 I10240, decode
              batches of 1/16/64/256 tokens (the stack's batch sizes)

Arrays are numpy; BF16 is carried as uint16 bit patterns.
"""
from __future__ import annotations

import dataclasses

import numpy as np

CONFIGS = {
    "c0": dict(hidden=256, experts=8, top_k=2, inter=128, shared_inter=128, tokens=16, scaling=1.0),
    "c1": dict(hidden=2048, experts=64, top_k=4, inter=1536, shared_inter=1536, tokens=64, scaling=2.5),
    "c2": dict(hidden=2048, experts=64, top_k=4, inter=1536, shared_inter=1536, tokens=8192, scaling=2.5),
    "c3": dict(hidden=2048, experts=64, top_k=4, inter=1536, shared_inter=1536, tokens=16384, scaling=2.5),
}
SWIGLU_LIMIT = 10.0  # model_spec swiglu_limit; the benchmark configs leave it unstated


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even F32 -> BF16 bit patterns (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def e4m3_encode_normal(v: np.ndarray) -> np.ndarray:
    """E4M3FN codes of positive values in the normal range [2^-6, 448]
    (round to nearest even, saturating at 448 = 0x7e)."""
    v = np.asarray(v, dtype=np.float32)
    f, ex = np.frexp(v)
    biased = ex.astype(np.int32) + 6
    mant = np.rint((f * np.float32(2) - np.float32(1)) * np.float32(8)).astype(np.int32)
    carry = mant == 8
    mant = np.where(carry, 0, mant)
    biased = biased + carry.astype(np.int32)
    sat = (biased > 15) | ((biased == 15) & (mant > 6))
    code = np.where(sat, 0x7E, (biased << 3) | mant)
    return code.astype(np.uint8)


@dataclasses.dataclass
class Layer:
    hidden: int
    experts: int
    top_k: int
    inter: int
    shared_inter: int
    scaling: float
    swiglu_limit: float
    bf16_experts: bool
    router_w: np.ndarray
    bias: np.ndarray
    shared_gate: np.ndarray | None
    shared_up: np.ndarray | None
    shared_down: np.ndarray | None
    # NVFP4 experts
    gate_packed: np.ndarray | None = None
    gate_scales: np.ndarray | None = None
    up_packed: np.ndarray | None = None
    up_scales: np.ndarray | None = None
    down_packed: np.ndarray | None = None
    down_scales: np.ndarray | None = None
    gate_ws2: np.ndarray | None = None
    gate_in: np.ndarray | None = None
    up_ws2: np.ndarray | None = None
    up_in: np.ndarray | None = None
    down_ws2: np.ndarray | None = None
    down_in: np.ndarray | None = None
    # BF16 experts (the layer-45 form)
    gate_bf16: np.ndarray | None = None
    up_bf16: np.ndarray | None = None
    down_bf16: np.ndarray | None = None

    def weight_bytes(self, active_experts: int | None = None) -> int:
        """Bytes of every weight a forward must stream (all experts unless
        `active_experts` is given)."""
        e = self.experts if active_experts is None else active_experts
        H, I, Is = self.hidden, self.inter, self.shared_inter
        per = (2 * I * H + H * I) * 2 if self.bf16_experts else (2 * I * H + H * I) // 2 + (2 * I * H + H * I) // 16
        return e * per + 3 * Is * H * 2 + self.experts * H * 2 + self.experts * 4


def _normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def _scales(rng: np.random.Generator, shape) -> np.ndarray:
    s = np.abs(rng.standard_normal(shape, dtype=np.float32))
    s = np.clip(s, np.float32(2.0 ** -6), np.float32(448.0))
    return e4m3_encode_normal(s)


def make_layer(cfg: dict, seed: int, bf16_experts: bool = False) -> Layer:
    rng = np.random.Generator(np.random.PCG64(seed))
    H, E, I, Is = cfg["hidden"], cfg["experts"], cfg["inter"], cfg["shared_inter"]
    router_w = f32_to_bf16_bits(_normal(rng, (E, H), 0.02))
    bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
    lay = Layer(hidden=H, experts=E, top_k=cfg["top_k"], inter=I, shared_inter=Is, scaling=float(cfg["scaling"]),
                swiglu_limit=SWIGLU_LIMIT, bf16_experts=bf16_experts, router_w=router_w, bias=bias,
                shared_gate=None, shared_up=None, shared_down=None)
    if bf16_experts:
        lay.gate_bf16 = f32_to_bf16_bits(_normal(rng, (E, I, H), 0.02))
        lay.up_bf16 = f32_to_bf16_bits(_normal(rng, (E, I, H), 0.02))
        lay.down_bf16 = f32_to_bf16_bits(_normal(rng, (E, H, I), 0.02))
    else:
        lay.gate_packed = rng.integers(0, 256, (E, I, H // 2), dtype=np.uint8)
        lay.gate_scales = _scales(rng, (E, I, H // 16))
        lay.up_packed = rng.integers(0, 256, (E, I, H // 2), dtype=np.uint8)
        lay.up_scales = _scales(rng, (E, I, H // 16))
        lay.down_packed = rng.integers(0, 256, (E, H, I // 2), dtype=np.uint8)
        lay.down_scales = _scales(rng, (E, H, I // 16))
        ws2 = np.full(E, np.float32(1) / np.float32(448), dtype=np.float32)
        ins = np.full(E, np.float32(1) / np.float32(6), dtype=np.float32)
        lay.gate_ws2, lay.up_ws2, lay.down_ws2 = ws2.copy(), ws2.copy(), ws2.copy()
        lay.gate_in, lay.up_in, lay.down_in = ins.copy(), ins.copy(), ins.copy()
    if Is > 0:
        lay.shared_gate = f32_to_bf16_bits(_normal(rng, (Is, H), 0.02))
        lay.shared_up = f32_to_bf16_bits(_normal(rng, (Is, H), 0.02))
        lay.shared_down = f32_to_bf16_bits(_normal(rng, (H, Is), 0.02))
    return lay


def make_tokens(cfg: dict, seed: int, tokens: int | None = None) -> np.ndarray:
    """x as BF16 bit patterns [T, H]."""
    rng = np.random.Generator(np.random.PCG64(seed + 1_000_003))
    T = cfg["tokens"] if tokens is None else tokens
    return f32_to_bf16_bits(rng.standard_normal((T, cfg["hidden"]), dtype=np.float32))


def _approx_choice(lay: Layer, x_bits: np.ndarray) -> np.ndarray:
    x = bf16_bits_to_f32(x_bits)
    w = bf16_bits_to_f32(lay.router_w)
    logits = x @ w.T
    return (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)


def balance_bias(lay: Layer, x_bits: np.ndarray, tol: float = 0.06, iters: int = 400) -> np.ndarray:
    """Tunes the correction bias until every expert receives T*k/E tokens
    within `tol` (approximate logits; the exact router lands within the
    benchmark's 10%)."""
    scores = _approx_choice(lay, x_bits)
    T, E, k = scores.shape[0], lay.experts, lay.top_k
    target = T * k / E
    bias = lay.bias.astype(np.float64).copy()
    for _ in range(iters):
        choice = scores + bias[None, :]
        top = np.argpartition(-choice, k - 1, axis=1)[:, :k]
        counts = np.bincount(top.ravel(), minlength=E)
        dev = (counts - target) / target
        if np.max(np.abs(dev)) <= tol:
            break
        bias -= 0.02 * np.clip(dev, -1.0, 1.0)
    return bias.astype(np.float32)


def zipf_bias(lay: Layer, s: float = 1.1, lam: float = 1.0) -> np.ndarray:
    """bias + lam * log p_e with p_e proportional to (e + 1)^-s."""
    e = np.arange(lay.experts, dtype=np.float64)
    p = (e + 1.0) ** (-s)
    p /= p.sum()
    return (lay.bias.astype(np.float64) + lam * np.log(p)).astype(np.float32)


# The log-prior weight at which c3's pick shares come closest to the Zipf(1.1)
# distribution itself (calibrate_zipf_lambda over its grid, seed 3).  At the
# literal lambda = 1 the prior (0 ... -4.6) swamps the sigmoid scores in (0, 1)
# and 93% of the picks land on experts 0-3, each of which then takes every
# token (a share of 1/k); at this lambda experts 0-3 take 48% of the picks
# (Zipf: 50%) and the busiest expert 18%.
C3_LAMBDA_CALIBRATED = 0.145


def calibrate_zipf_lambda(lay: Layer, x_bits: np.ndarray, s: float = 1.1,
                          grid: np.ndarray | None = None) -> float:
    """The lambda on `grid` (default 0, 0.005, ..., 1) whose routing puts the
    share of picks per expert closest, in L1 distance, to p_e proportional to
    (e + 1)^-s.  `lay.bias` is the bias before the prior; the routing uses the
    approximate scores of balance_bias (selection only, which is all the
    shares need)."""
    grid = np.round(np.arange(0.0, 1.0 + 1e-9, 0.005), 3) if grid is None else grid
    scores = _approx_choice(lay, x_bits)
    E, k = lay.experts, lay.top_k
    e = np.arange(E, dtype=np.float64)
    p = (e + 1.0) ** (-s)
    p /= p.sum()
    base = lay.bias.astype(np.float64)
    best, best_l1 = float(grid[0]), np.inf
    for lam in grid:
        choice = scores + (base + lam * np.log(p))[None, :]
        top = np.argpartition(-choice, k - 1, axis=1)[:, :k]
        share = np.bincount(top.ravel(), minlength=E) / top.size
        l1 = float(np.abs(share - p).sum())
        if l1 < best_l1:
            best, best_l1 = float(lam), l1
    return best


def config_layer(name: str, seed: int | None = None, bf16_experts: bool = False,
                 zipf_lambda: float = 1.0) -> tuple[Layer, np.ndarray]:
    """The layer and the token batch of a named configuration (`zipf_lambda`
    weights c3's log-prior)."""
    cfg = CONFIGS[name]
    seed = {"c0": 0, "c1": 1, "c2": 2, "c3": 3}[name] if seed is None else seed
    lay = make_layer(cfg, seed, bf16_experts=bf16_experts)
    x = make_tokens(cfg, seed)
    if name == "c2":
        lay.bias = balance_bias(lay, x)
    elif name == "c3":
        lay.bias = zipf_bias(lay, lam=zipf_lambda)
    return lay, x


DENSE_CONFIGS = {
    "c4_dense": dict(hidden=2048, inter=10240, tokens=64),
}


@dataclasses.dataclass
class DenseLayer:
    """The dense NVFP4 MLP of one of the first layers (mlp.{gate,up,down}_proj)."""
    hidden: int
    inter: int
    swiglu_limit: float
    gate_packed: np.ndarray   # [I, H/2]
    gate_scales: np.ndarray   # [I, H/16]
    up_packed: np.ndarray
    up_scales: np.ndarray
    down_packed: np.ndarray   # [H, I/2]
    down_scales: np.ndarray   # [H, I/16]
    gate_ws2: float = 1.0 / 448.0
    gate_in: float = 1.0 / 6.0
    up_ws2: float = 1.0 / 448.0
    up_in: float = 1.0 / 6.0
    down_ws2: float = 1.0 / 448.0
    down_in: float = 1.0 / 6.0

    def weight_bytes(self) -> int:
        """Bytes a forward streams: E2M1 codes plus E4M3 block scales."""
        n = 3 * self.inter * self.hidden
        return n // 2 + n // 16


def make_dense_layer(hidden: int, inter: int, seed: int) -> DenseLayer:
    """NVFP4 weights with the same distributions as the routed experts."""
    rng = np.random.Generator(np.random.PCG64(seed))
    H, I = hidden, inter
    f32 = lambda v: float(np.float32(v))  # noqa: E731
    return DenseLayer(
        hidden=H, inter=I, swiglu_limit=SWIGLU_LIMIT,
        gate_packed=rng.integers(0, 256, (I, H // 2), dtype=np.uint8), gate_scales=_scales(rng, (I, H // 16)),
        up_packed=rng.integers(0, 256, (I, H // 2), dtype=np.uint8), up_scales=_scales(rng, (I, H // 16)),
        down_packed=rng.integers(0, 256, (H, I // 2), dtype=np.uint8), down_scales=_scales(rng, (H, I // 16)),
        gate_ws2=f32(np.float32(1) / np.float32(448)), gate_in=f32(np.float32(1) / np.float32(6)),
        up_ws2=f32(np.float32(1) / np.float32(448)), up_in=f32(np.float32(1) / np.float32(6)),
        down_ws2=f32(np.float32(1) / np.float32(448)), down_in=f32(np.float32(1) / np.float32(6)))


# ---- the synthetic decoder stack of configs[4] --------------------------------
STACK_CONFIGS = {
    # layers 0-2 dense NVFP4 MLPs (H2048, I10240), layers 3-44 NVFP4
    # MoE layers as in c1, layer 45 BF16 routed experts; BF16 GQA attention
    # 32 q heads / 4 KV heads / dim 128; vocab 151552; 2048-token context
    "c4": dict(vocab=151552, hidden=2048, layers=46, dense_layers=3, bf16_expert_layers=1, dense_inter=10240,
               experts=64, top_k=4, inter=1536, shared_inter=1536, scaling=2.5, q_heads=32, kv_heads=4,
               context=2048),
    # a small stack with the same structure, for parity against the CPU oracle
    "tiny": dict(vocab=1000, hidden=256, layers=4, dense_layers=1, bf16_expert_layers=1, dense_inter=512,
                 experts=8, top_k=2, inter=128, shared_inter=128, scaling=1.0, q_heads=8, kv_heads=1,
                 context=1024),
}
STACK_BATCHES = (1, 16, 64, 256)  # configs[4]'s greedy-decode batch sizes


@dataclasses.dataclass
class StackLayer:
    wq: np.ndarray          # BF16 [q_heads 128, H]
    wk: np.ndarray          # BF16 [kv_heads 128, H]
    wv: np.ndarray          # BF16 [kv_heads 128, H]
    wo: np.ndarray          # BF16 [H, q_heads 128]
    attn_norm: np.ndarray   # F32 [H]
    ffn_norm: np.ndarray    # F32 [H]
    q_norm: np.ndarray      # F32 [128]
    k_norm: np.ndarray      # F32 [128]
    ffn: object             # DenseLayer or Layer (NVFP4 or BF16 experts)


@dataclasses.dataclass
class StackModel:
    cfg: dict
    embed: np.ndarray       # BF16 [vocab, H], ~N(0, 1)
    lm_head: np.ndarray     # BF16 [vocab, H], ~N(0, 0.02)
    final_norm: np.ndarray  # F32 [H]
    layers: list


def make_stack(cfg: dict, seed: int, share: bool = False) -> StackModel:
    """Random-init weights of the stack (BF16 ~N(0, 0.02) projections, NVFP4
    experts as make_layer, norms 1 + N(0, 0.05)).  share=True generates one
    attention block, one dense MLP and one MoE layer and lists them for every
    layer of their kind (each layer still gets its own device copy when
    bound): the full configuration's 16 GB of weights without generating
    them 46 times on the host."""
    rng = np.random.Generator(np.random.PCG64(seed))
    H, V = cfg["hidden"], cfg["vocab"]
    nq, nkv, D = cfg["q_heads"], cfg["kv_heads"], 128

    def attn(r):
        return dict(wq=f32_to_bf16_bits(_normal(r, (nq * D, H), 0.02)),
                    wk=f32_to_bf16_bits(_normal(r, (nkv * D, H), 0.02)),
                    wv=f32_to_bf16_bits(_normal(r, (nkv * D, H), 0.02)),
                    wo=f32_to_bf16_bits(_normal(r, (H, nq * D), 0.02)),
                    attn_norm=(1 + _normal(r, (H,), 0.05)).astype(np.float32),
                    ffn_norm=(1 + _normal(r, (H,), 0.05)).astype(np.float32),
                    q_norm=(1 + _normal(r, (D,), 0.05)).astype(np.float32),
                    k_norm=(1 + _normal(r, (D,), 0.05)).astype(np.float32))

    moe_cfg = dict(hidden=H, experts=cfg["experts"], top_k=cfg["top_k"], inter=cfg["inter"],
                   shared_inter=cfg["shared_inter"], scaling=cfg["scaling"])
    L, nd, nb = cfg["layers"], cfg["dense_layers"], cfg["bf16_expert_layers"]
    shared_attn = attn(rng) if share else None
    shared_dense = make_dense_layer(H, cfg["dense_inter"], seed + 7) if share and nd else None
    shared_moe = make_layer(moe_cfg, seed + 11) if share and L - nd - nb > 0 else None
    layers = []
    for l in range(L):
        a = shared_attn if share else attn(rng)
        if l < nd:
            f = shared_dense if share else make_dense_layer(H, cfg["dense_inter"], seed + 100 + l)
        elif l >= L - nb:
            f = make_layer(moe_cfg, seed + 100 + l, bf16_experts=True)
        else:
            f = shared_moe if share else make_layer(moe_cfg, seed + 100 + l)
        layers.append(StackLayer(ffn=f, **a))
    embed = f32_to_bf16_bits(rng.standard_normal((V, H), dtype=np.float32))
    lm_head = f32_to_bf16_bits(_normal(rng, (V, H), 0.02))
    final_norm = (1 + _normal(rng, (H,), 0.05)).astype(np.float32)
    return StackModel(cfg=cfg, embed=embed, lm_head=lm_head, final_norm=final_norm, layers=layers)
