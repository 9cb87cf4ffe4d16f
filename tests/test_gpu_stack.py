"""The decoder stack's greedy step (nf_stack_*) against the CPU oracle
(oracle/stack_oracle.py: the pinned C primitives composed with a restatement
of the reference's GQA attention math) on a small stack of the benchmark's
structure -- a dense NVFP4 MLP layer, two NVFP4 MoE layers, a BF16-expert
MoE layer -- with a loaded KV history of different lengths per sequence.

Tolerance: the stack's projections take BF16 inputs (tensor cores) where the
oracle's gemv takes F32, and the caches hold BF16; the final hidden state
must agree within max-abs 5e-2 and cosine 0.9995, and every greedy token
whose oracle margin (best minus second logit) exceeds 0.02 must be equal."""
from pathlib import Path

import numpy as np
import pytest

from helpers import REPO, assert_close, load_module, nfm, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
m, wl = nfm(), workload()
so = load_module("nf_stack_oracle", REPO / "oracle" / "stack_oracle.py")


def make_stack(model, max_batch, max_context):
    c = model.cfg
    st = m.DecoderStack(vocab=c["vocab"], hidden=c["hidden"], layers=c["layers"], dense_layers=c["dense_layers"],
                        bf16_expert_layers=c["bf16_expert_layers"], dense_inter=c["dense_inter"],
                        experts=c["experts"], top_k=c["top_k"], inter=c["inter"], shared_inter=c["shared_inter"],
                        routed_scaling=c["scaling"], q_heads=c["q_heads"], kv_heads=c["kv_heads"],
                        max_batch=max_batch, max_context=max_context)
    st.bind_model(model)
    return st


def load_history(st, model, positions, max_batch, L, seed):
    """Random BF16 keys and values at positions < positions[i] of every layer's
    cache, on the GPU and (as F32) for the oracle."""
    rng = np.random.default_rng(seed)
    nkv = model.cfg["kv_heads"]
    k_hist, v_hist = [], []
    for l in range(len(model.layers)):
        kb = wl.f32_to_bf16_bits(rng.standard_normal((max_batch, nkv, L, 128), dtype=np.float32))
        vb = wl.f32_to_bf16_bits(rng.standard_normal((max_batch, nkv, L, 128), dtype=np.float32))
        for i, p in enumerate(positions):
            kb[i, :, p:] = 0
            vb[i, :, p:] = 0
        st.load_kv(l, kb, vb)
        k_hist.append(so.bf16_bits_to_f32(kb).copy())
        v_hist.append(so.bf16_bits_to_f32(vb).copy())
    return k_hist, v_hist


def check_step(st, model, tokens, positions, k_hist, v_hist):
    B = len(tokens)
    H = model.cfg["hidden"]
    tok = torch.from_numpy(np.asarray(tokens, np.int32)).cuda()
    pos = torch.from_numpy(np.asarray(positions, np.int32)).cuda()
    nxt = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    fin = torch.empty((B, H), dtype=torch.float32, device="cuda")
    st.decode(tok, pos, B, nxt, fin)
    st.sync()
    want_next, logits, want_fin = so.decode_step(model, k_hist, v_hist, np.asarray(tokens), np.asarray(positions))
    got_fin = fin.cpu().numpy()
    assert_close(got_fin, want_fin, max_abs=5e-2, min_cos=0.9995, what="final hidden state")
    got_next = nxt.cpu().numpy()
    srt = np.sort(logits, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    clear = margin > 0.02
    assert clear.sum() >= max(1, B // 2)
    assert np.array_equal(got_next[clear], want_next[clear]), (got_next, want_next, margin)
    return got_next


@pytest.mark.parametrize("batch", [3, 40])
def test_stack_greedy_steps_match_oracle(batch):
    cfg = wl.STACK_CONFIGS["tiny"]
    model = wl.make_stack(cfg, seed=5)
    L = cfg["context"]
    rng = np.random.default_rng(batch)
    positions = rng.integers(0, L - 2, batch)
    positions[0] = 0            # an empty history
    positions[-1] = L - 2       # the whole cache (the next step writes the last slot)
    st = make_stack(model, batch, L)
    k_hist, v_hist = load_history(st, model, positions, batch, L, seed=batch)
    tokens = rng.integers(0, cfg["vocab"], batch)
    nxt = check_step(st, model, tokens, positions, k_hist, v_hist)
    # the next step feeds the greedy tokens back one position later
    check_step(st, model, nxt, positions + 1, k_hist, v_hist)
    st.close()


def test_stack_rejects_bad_tokens_and_positions():
    cfg = wl.STACK_CONFIGS["tiny"]
    model = wl.make_stack(cfg, seed=6)
    st = make_stack(model, 2, 64)
    tok = torch.tensor([1, cfg["vocab"]], dtype=torch.int32, device="cuda")  # the second is outside
    pos = torch.tensor([0, 0], dtype=torch.int32, device="cuda")
    nxt = torch.empty(2, dtype=torch.int32, device="cuda")
    st.decode(tok, pos, 2, nxt)
    with pytest.raises(m.NfError, match="outside the vocabulary"):
        st.sync()
    tok = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    pos = torch.tensor([0, 64], dtype=torch.int32, device="cuda")  # beyond max_context
    st.decode(tok, pos, 2, nxt)
    with pytest.raises(m.NfError, match="outside the cache"):
        st.sync()
    st.close()
