"""The oracle reproduces the reference's committed outputs on the seeded
tiny configuration (tests/golden/c0_reference.npz, made by
tests/golden/make_golden.py from the reference's own sources)."""
from pathlib import Path

import numpy as np
import pytest

from golden.make_golden import input_digest, digest, residual_for
from helpers import oracle, workload

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "c0_reference.npz")
orc, wl = oracle(), workload()


@pytest.mark.parametrize("tag,bf16", [("nvfp4", False), ("bf16", True)])
def test_inputs_pinned(tag, bf16):
    lay, x_bits = wl.config_layer("c0", bf16_experts=bf16)
    assert input_digest(lay, x_bits) == str(GOLDEN[f"{tag}_inputs_sha256"]), "synthetic input generator changed"
    assert digest(residual_for(x_bits)) == str(GOLDEN[f"{tag}_residual_sha256"])


@pytest.mark.parametrize("tag,bf16", [("nvfp4", False), ("bf16", True)])
def test_port_matches_reference_golden(tag, bf16):
    lay, x_bits = wl.config_layer("c0", bf16_experts=bf16)
    x = wl.bf16_bits_to_f32(x_bits)
    y, idx, w = orc.moe_layer(orc.port(), lay, x)
    assert np.array_equal(idx, GOLDEN[f"{tag}_idx"])
    assert np.array_equal(w.view(np.uint32), GOLDEN[f"{tag}_w"].view(np.uint32))
    assert np.array_equal(y.view(np.uint32), GOLDEN[f"{tag}_y"].view(np.uint32))
    yr, _, _ = orc.moe_layer(orc.port(), lay, x, residual_for(x_bits))
    assert np.array_equal(yr.view(np.uint32), GOLDEN[f"{tag}_y_residual"].view(np.uint32))


def test_port_quantiser_matches_reference_golden():
    lay, x_bits = wl.config_layer("c0")
    x = wl.bf16_bits_to_f32(x_bits)
    fake, _, _ = orc.quant_codes(orc.port(), x, float(lay.gate_in[0]))
    assert np.array_equal(fake.view(np.uint32), GOLDEN["quant_fake"].view(np.uint32))


def test_dense_inputs_pinned_and_port_matches_reference_golden():
    """The dense MLP (dense_mlp, src/text_forward.cpp:909-915): the seeded
    inputs are the ones the golden file was made from, and the restatement
    gives the reference's bits with and without the residual."""
    from golden.make_golden import dense_case, dense_digest

    g = np.load(Path(__file__).resolve().parent / "golden" / "dense_reference.npz")
    lay, x_bits, res = dense_case()
    assert dense_digest(lay, x_bits) == str(g["inputs_sha256"]), "dense input generator changed"
    assert digest(res) == str(g["residual_sha256"])
    x = wl.bf16_bits_to_f32(x_bits)
    assert np.array_equal(orc.dense_mlp(orc.port(), lay, x).view(np.uint32), g["y"].view(np.uint32))
    assert np.array_equal(orc.dense_mlp(orc.port(), lay, x, res).view(np.uint32), g["y_residual"].view(np.uint32))
