"""Generates the golden files from the reference's own outputs (oracle/_ref,
compiled from the reference's sources), with SHA-256 pins of the generated
inputs:
  c0_reference.npz     the MoE layer on the seeded tiny configuration c0
  dense_reference.npz  the dense NVFP4 MLP (dense_mlp) on a seeded small shape

Run in a container that holds the reference tree:
    python tests/golden/make_golden.py            # both files
    python tests/golden/make_golden.py dense      # the dense file only
The GPU box has no reference tree; tests compare against these files there.
"""
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from helpers import oracle, workload  # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def input_digest(lay, x_bits) -> str:
    return digest(x_bits, lay.router_w, lay.bias, lay.gate_packed, lay.gate_scales, lay.up_packed, lay.up_scales,
                  lay.down_packed, lay.down_scales, lay.gate_ws2, lay.gate_in, lay.up_ws2, lay.up_in, lay.down_ws2,
                  lay.down_in, lay.gate_bf16, lay.up_bf16, lay.down_bf16, lay.shared_gate, lay.shared_up,
                  lay.shared_down)


def residual_for(x_bits):
    rng = np.random.Generator(np.random.PCG64(4242))
    return rng.standard_normal(x_bits.shape).astype(np.float32)


def main():
    orc, wl = oracle(), workload()
    ref = orc.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libnf_ref.so is missing: run make -C oracle with the reference tree present")
    out = {}
    for tag, bf16 in (("nvfp4", False), ("bf16", True)):
        lay, x_bits = wl.config_layer("c0", bf16_experts=bf16)
        x = wl.bf16_bits_to_f32(x_bits)
        res = residual_for(x_bits)
        y, idx, w = orc.moe_layer(ref, lay, x)
        yr, _, _ = orc.moe_layer(ref, lay, x, res)
        out[f"{tag}_inputs_sha256"] = np.array(input_digest(lay, x_bits))
        out[f"{tag}_residual_sha256"] = np.array(digest(res))
        out[f"{tag}_y"] = y
        out[f"{tag}_y_residual"] = yr
        out[f"{tag}_idx"] = idx
        out[f"{tag}_w"] = w
    # quantiser vectors: reference fake-quant output on the c0 tokens
    lay, x_bits = wl.config_layer("c0")
    x = wl.bf16_bits_to_f32(x_bits)
    q = np.zeros_like(x)
    for r in range(x.shape[0]):
        assert ref.ref_quant_dequant(orc.p(x[r]), x.shape[1], float(lay.gate_in[0]), orc.p(q[r])) == 0
    out["quant_fake"] = q
    np.savez_compressed(HERE / "c0_reference.npz", **out)
    print("wrote", HERE / "c0_reference.npz")


DENSE_SHAPE = dict(hidden=256, inter=512, tokens=16, seed=40)


def dense_case():
    """The dense golden case: (layer, token bits, residual)."""
    wl = workload()
    c = DENSE_SHAPE
    lay = wl.make_dense_layer(c["hidden"], c["inter"], c["seed"])
    x_bits = wl.make_tokens(dict(hidden=c["hidden"], tokens=c["tokens"]), c["seed"])
    return lay, x_bits, residual_for(x_bits)


def dense_digest(lay, x_bits) -> str:
    return digest(x_bits, lay.gate_packed, lay.gate_scales, lay.up_packed, lay.up_scales, lay.down_packed,
                  lay.down_scales, np.array([lay.gate_ws2, lay.gate_in, lay.up_ws2, lay.up_in, lay.down_ws2,
                                             lay.down_in], np.float32))


def main_dense():
    orc, wl = oracle(), workload()
    ref = orc.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libnf_ref.so is missing: run make -C oracle with the reference tree present")
    lay, x_bits, res = dense_case()
    x = wl.bf16_bits_to_f32(x_bits)
    out = {"inputs_sha256": np.array(dense_digest(lay, x_bits)), "residual_sha256": np.array(digest(res)),
           "y": orc.dense_mlp(ref, lay, x), "y_residual": orc.dense_mlp(ref, lay, x, res)}
    np.savez_compressed(HERE / "dense_reference.npz", **out)
    print("wrote", HERE / "dense_reference.npz")


if __name__ == "__main__":
    if sys.argv[1:] != ["dense"]:
        main()
    main_dense()
