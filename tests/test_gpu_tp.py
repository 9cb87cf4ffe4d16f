"""Tensor-parallel BF16 linears (nf_tp_*): the GPU form of the reference's
row split + gather_rows (src/text_forward.cpp:242-256, 803-830).

Every output is checked bit for bit against the oracle's gemv_bf16 (a
restatement pinned to the reference's own gemv_bf16): on one GPU over ragged
shapes, special values and the lm_head's [151552, 2048] shape; and on two
GPUs and on every GPU of the box, each rank holding only its row block, over
both transports (NVLink peer stores and NCCL).  The greedy pick is checked
against a restatement of the reference's argmax scan (ties, NaN)."""
import os
import socket
import sys

import numpy as np
import pytest

from helpers import REPO, nfm, oracle, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
m, orc, wl = nfm(), oracle(), workload()


def gemv_oracle(w_bits: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y [T, rows] = gemv_bf16(W, x_t) for every token (the oracle port)."""
    lib = orc.port()
    rows, cols = w_bits.shape
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    out = np.zeros((x.shape[0], rows), np.float32)
    for t in range(x.shape[0]):
        xt = np.ascontiguousarray(x[t], dtype=np.float32)
        lib.or_gemv_bf16(orc.p(w), orc.p(xt), rows, cols, 0, rows, orc.p(out[t]))
    return out


def same_bits(got: np.ndarray, want: np.ndarray) -> bool:
    """Bit-equal, except that a NaN only has to be a NaN: the GPU writes the
    canonical NaN where the x86 reference keeps an operand's payload and sign
    (or makes the negative default NaN), which is platform behaviour, not a
    result."""
    gn, wn = np.isnan(got), np.isnan(want)
    return bool(np.array_equal(gn, wn) and np.array_equal(got.view(np.uint32)[~gn], want.view(np.uint32)[~wn]))


def argmax_ref(logits: np.ndarray) -> np.ndarray:
    """TextModel::argmax's scan (src/text_forward.cpp:668-681): best = row 0,
    replaced only by a strictly greater value."""
    out = np.zeros(logits.shape[0], np.int32)
    for t, row in enumerate(logits):
        if np.isnan(row[0]):
            continue
        ok = ~np.isnan(row)
        best = np.max(row[ok])
        out[t] = int(np.nonzero(ok & (row == best))[0][0])
    return out


def make_case(rows: int, cols: int, tokens: int, seed: int):
    rng = np.random.default_rng(seed)
    w = wl.f32_to_bf16_bits(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((tokens, cols), dtype=np.float32)
    return w, x


def run_one_gpu(w, x, tp=None, y_out=True):
    rows, cols = w.shape
    T = x.shape[0]
    own = tp is None
    tp = tp or m.TpGroup(max_tokens=max(T, 1), max_rows=rows)
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.full((T, rows), float("nan"), device="cuda") if y_out else None
    tp.linear_bf16(wd, rows, cols, xd, T, y)
    tp.sync()
    out = y.cpu().numpy() if y_out else None
    if own:
        tp.close()
    return out


@pytest.mark.parametrize("rows,cols,tokens", [(1000, 256, 1), (1000, 256, 3), (777, 260, 8), (513, 2048, 17),
                                              (256, 4096, 64)])
def test_linear_bit_exact_one_gpu(rows, cols, tokens):
    w, x = make_case(rows, cols, tokens, seed=rows + cols + tokens)
    got = run_one_gpu(w, x)
    want = gemv_oracle(w, x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_linear_special_values_bit_exact():
    """Infinities, NaN, signed zeros, subnormals and huge values in x and W
    follow the reference's separately rounded products and sums."""
    w, x = make_case(300, 128, 5, seed=3)
    x[0, 5] = np.inf
    x[1, 7] = np.nan
    x[2, :] = -0.0
    x[3, 9] = np.float32(1e-40)
    x[4, 11] = np.float32(3e38)
    w[17, :] = 0x8000  # -0.0 row
    w[18, 3] = 0x7F80  # +inf
    w[19, 4] = 0x0001  # BF16 subnormal
    got = run_one_gpu(w, x)
    want = gemv_oracle(w, x)
    assert np.isnan(want).any() and np.isinf(want).any()
    assert same_bits(got, want)


def test_lm_head_shape_and_greedy_pick():
    """The lm_head's [151552, 2048] at 1 and 4 tokens: logits bit-exact and the
    greedy tokens equal the reference scan's."""
    rows, cols = 151552, 2048
    w, x = make_case(rows, cols, 4, seed=11)
    tp = m.TpGroup(max_tokens=4, max_rows=rows)
    for T in (1, 4):
        got = run_one_gpu(w, x[:T], tp)
        want = gemv_oracle(w, x[:T])
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        idx = torch.empty(T, dtype=torch.int32, device="cuda")
        tp.argmax(T, rows, idx)
        tp.sync()
        assert np.array_equal(idx.cpu().numpy(), argmax_ref(want))
    tp.close()


def test_argmax_ties_and_nan():
    """Equal maxima: the lowest row; a NaN row never wins; +0 and -0 tie; a NaN
    in row 0 is kept.  (A NaN weight makes its row NaN for every token.)"""
    rows, cols = 64, 4
    one = wl.f32_to_bf16_bits(np.array([1.0], np.float32))[0]
    w = np.zeros((rows, cols), np.uint16)
    w[:, 0] = one      # every row: x[t, 0]
    w[10, 1] = one     # rows 10 and 40: + x[t, 1]
    w[40, 1] = one
    w[20, 2] = 0x7FC0  # row 20: NaN
    w[33, 3] = one     # row 33: + x[t, 3]
    x = np.array([[0.0, 2.0, 0.0, 0.0],    # rows 10 and 40 tie at 2: row 10
                  [-1.0, 0.0, 0.0, 0.0],   # every row -1: row 0
                  [0.0, 0.0, 0.0, 5.0],    # row 33
                  [0.0, 0.0, 0.0, -5.0],   # row 33 at -5, the rest 0: row 0
                  [-0.0, 0.0, 0.0, 0.0]],  # +0 everywhere: row 0
                 np.float32)
    tp = m.TpGroup(max_tokens=5, max_rows=rows)
    got = run_one_gpu(w, x, tp)
    want = gemv_oracle(w, x)
    assert same_bits(got, want)
    idx = torch.empty(5, dtype=torch.int32, device="cuda")
    tp.argmax(5, rows, idx)
    tp.sync()
    assert list(idx.cpu().numpy()) == list(argmax_ref(want)) == [10, 0, 33, 0, 0]
    w[0, 2] = 0x7FC0   # row 0 NaN: never replaced
    got = run_one_gpu(w, x, tp)
    tp.argmax(5, rows, idx)
    tp.sync()
    assert list(idx.cpu().numpy()) == list(argmax_ref(gemv_oracle(w, x))) == [0, 0, 0, 0, 0]
    tp.close()


def test_consecutive_calls_and_capacity():
    """Calls in a row alternate the gather buffers: each result stays right;
    zero tokens is a no-op; sizes beyond the handle are refused."""
    tp = m.TpGroup(max_tokens=8, max_rows=2048)
    for i in range(5):
        w, x = make_case(2048 - 100 * i, 512, 1 + i, seed=40 + i)
        got = run_one_gpu(w, x, tp)
        assert np.array_equal(got.view(np.uint32), gemv_oracle(w, x).view(np.uint32))
    wd = torch.zeros((16, 512), dtype=torch.int16, device="cuda")
    xd = torch.zeros((9, 512), dtype=torch.float32, device="cuda")
    tp.linear_bf16(wd, 16, 512, xd, 0)
    with pytest.raises(m.NfError, match="max_tokens"):
        tp.linear_bf16(wd, 16, 512, xd, 9)
    with pytest.raises(m.NfError, match="max_rows"):
        tp.linear_bf16(torch.zeros((4096, 512), dtype=torch.int16, device="cuda"), 4096, 512, xd, 1)
    with pytest.raises(m.NfError, match="multiple of 4"):
        tp.linear_bf16(wd, 16, 510, xd, 1)
    tp.sync()
    tp.close()


# ---- several GPUs ------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out_dir: str, transport: str) -> None:
    sys.path.insert(0, str(REPO / "tests"))
    os.environ["NF_TP_TRANSPORT"] = transport
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    mm = nfm()
    gid = [mm.ep_group_id() if rank == 0 else None]
    dist.broadcast_object_list(gid, src=0)
    shapes = [(1000, 256, 3), (151552, 2048, 2), (7, 64, 1), (4099, 512, 9)]  # (rows < world: a rank with no rows)
    tp = mm.TpGroup(max_tokens=9, max_rows=151552, rank=rank, world=world, group_id=gid[0], device=rank)
    res = {"transport": np.array(tp.transport())}
    s = torch.cuda.Stream()
    for i, (rows, cols, T) in enumerate(shapes):
        w, x = make_case(rows, cols, T, seed=100 + i)
        r0, r1 = tp.split(rows)
        wd = torch.from_numpy(np.ascontiguousarray(w[r0:r1]).view(np.int16)).cuda()
        xd = torch.from_numpy(x).cuda()
        y = torch.full((T, rows), float("nan"), device="cuda")
        idx = torch.empty(T, dtype=torch.int32, device="cuda")
        tp.linear_bf16(wd, rows, cols, xd, T, y, stream=s.cuda_stream)
        tp.argmax(T, rows, idx, stream=s.cuda_stream)
        tp.sync(s.cuda_stream)
        res[f"y{i}"] = y.cpu().numpy()
        res[f"i{i}"] = idx.cpu().numpy()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), **res)
    dist.barrier()  # every rank's last call is done before any handle of the group goes
    tp.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nvlink", "nccl"])
@pytest.mark.parametrize("ranks", ["two", "all"])
def test_tp_group_matches_one_rank(tmp_path, transport, ranks):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2 if ranks == "two" else min(n, 8)
    if ranks == "all" and world == 2:
        pytest.skip("only two GPUs: covered by the two-rank case")
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path), transport), nprocs=world,
                       start_method="spawn", join=True)
    got = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    assert all(str(g["transport"]) == transport for g in got)
    shapes = [(1000, 256, 3), (151552, 2048, 2), (7, 64, 1), (4099, 512, 9)]
    for i, (rows, cols, T) in enumerate(shapes):
        w, x = make_case(rows, cols, T, seed=100 + i)
        want = gemv_oracle(w, x)
        for g in got:  # every rank holds the whole output, bit for bit
            assert np.array_equal(g[f"y{i}"].view(np.uint32), want.view(np.uint32)), (i, rows)
            assert np.array_equal(g[f"i{i}"], argmax_ref(want))
