"""Expert parallelism on the CPU: the (destination, token, pick) exchange
layout, and the whole EP decomposition run by two and four gloo ranks -- route own
tokens, send rows to the owners of the picked experts, run the experts there
(the oracle's expert_forward), send the outputs back, combine in pick order --
against the single-rank oracle layer, bit for bit."""
import os
import socket
import sys

import numpy as np
import pytest

from helpers import PKG, REPO, load_module, oracle, workload

plan = load_module("nf_ep_plan", PKG / "ep_plan.py")


def test_owner_blocks():
    assert list(plan.owner(np.arange(8), 8, 2)) == [0, 0, 0, 0, 1, 1, 1, 1]
    assert list(plan.owner(np.arange(64), 64, 8)[::8]) == list(range(8))
    with pytest.raises(ValueError):
        plan.owner(np.arange(6), 6, 4)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_pack_is_destination_token_pick_order(world):
    rng = np.random.default_rng(world)
    T, K, E = 37, 4, 64
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    sp = plan.pack(idx, E, world)
    dest = plan.owner(idx, E, world)
    # brute force: sort (dest, t, p)
    keys = sorted((int(dest[t, p]), t, p) for t in range(T) for p in range(K))
    for s, (d, t, p) in enumerate(keys):
        assert sp.slot[t, p] == s
        assert sp.send_token[s] == t
        assert sp.send_expert[s] == idx[t, p] - d * (E // world)
    assert list(sp.counts) == [int((dest == d).sum()) for d in range(world)]
    assert sp.offsets[-1] == T * K
    assert sorted(sp.slot.ravel()) == list(range(T * K))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(dist, send: list, recv_shapes: list, dtype, rank: int, world: int) -> list:
    """Point-to-point exchange: send[p] to rank p, receive from every rank."""
    import torch

    out = [None] * world
    reqs = []
    for p in range(world):
        if p == rank:
            out[p] = send[p].copy()
            continue
        buf = torch.empty(recv_shapes[p], dtype=dtype)
        out[p] = buf
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(send[p])), p))
        reqs.append(dist.irecv(buf, p))
    for r in reqs:
        r.wait()
    return [o if isinstance(o, np.ndarray) else o.numpy() for o in out]


def _ep_rank(rank: int, world: int, port: int, out_dir: str, transport: str) -> None:
    sys.path.insert(0, str(REPO / "tests"))
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    wl, orc = workload(), oracle()
    lay, x_bits = wl.config_layer("c0")
    x_all = wl.bf16_bits_to_f32(x_bits)
    T_all, H, E, K = x_all.shape[0], lay.hidden, lay.experts, lay.top_k
    per_tok = T_all // world
    x = x_all[rank * per_tok:(rank + 1) * per_tok]
    # 1. route own tokens; the shared expert of own tokens (tap of the port layer)
    _, idx, w = orc.route_tokens(lay, x)
    _, _, _, _, shared = orc.moe_layer(orc.port(), lay, x, taps=True)
    # 2. send rows to the experts' owners in (destination, token, pick) order
    sp = plan.pack(idx, E, world)
    rows = x[sp.send_token]
    base = rank * (E // world)
    if transport == "nccl":
        # counts first, then exactly the rows that exist (the NCCL transport)
        counts = _exchange(dist, [np.array([c], np.int64) for c in sp.counts], [(1,)] * world, torch.int64, rank, world)
        rc = np.array([int(c[0]) for c in counts])
        send_rows = [rows[sp.offsets[p]:sp.offsets[p + 1]] for p in range(world)]
        send_e = [sp.send_expert[sp.offsets[p]:sp.offsets[p + 1]] for p in range(world)]
        recv_rows = _exchange(dist, send_rows, [(int(c), H) for c in rc], torch.float32, rank, world)
        recv_e = _exchange(dist, send_e, [(int(c),) for c in rc], torch.int64, rank, world)
        # 3. the owned experts on the received rows
        outs = []
        for p in range(world):
            o = np.zeros((rc[p], H), np.float32)
            for i in range(rc[p]):
                o[i] = orc.expert_forward(lay, base + int(recv_e[p][i]), recv_rows[p][i])[1]
            outs.append(o)
        # 4. outputs back to their sources, in send order
        back = _exchange(dist, outs, [(int(c), H) for c in sp.counts], torch.float32, rank, world)
        ret = np.concatenate(back) if back else np.zeros((0, H), np.float32)
    else:
        # the NVLink mailbox layout: fixed [cap] slots per source, each with its
        # count and the sender's offset; unused slots carry expert -1
        cap = per_tok * K
        boxes = []
        for p in range(world):
            lo, n = int(sp.offsets[p]), int(sp.counts[p])
            blk_rows = np.zeros((cap, H), np.float32)
            blk_e = np.full(cap + 2, -1, np.int64)  # [experts..., count, offset]
            blk_rows[:n] = rows[lo:lo + n]
            blk_e[:n] = sp.send_expert[lo:lo + n]
            blk_e[cap], blk_e[cap + 1] = n, lo
            boxes.append((blk_rows, blk_e))
        mb_rows = _exchange(dist, [b[0] for b in boxes], [(cap, H)] * world, torch.float32, rank, world)
        mb_e = _exchange(dist, [b[1] for b in boxes], [(cap + 2,)] * world, torch.int64, rank, world)
        # 3. the owned experts over every slot, empty ones skipped; outputs go
        #    back to each source at its own send positions
        outs = []
        for s in range(world):
            n, off = int(mb_e[s][cap]), int(mb_e[s][cap + 1])
            o = np.zeros((cap, H), np.float32)
            for j in range(cap):
                e = int(mb_e[s][j])
                if e < 0:
                    assert j >= n
                    continue
                o[j] = orc.expert_forward(lay, base + e, mb_rows[s][j])[1]
            head = np.zeros((1, H), np.float32)  # the sender's offset and count travel with the block
            head[0, 0], head[0, 1] = off, n
            outs.append(np.concatenate([head, o]))
        back = _exchange(dist, outs, [(cap + 1, H)] * world, torch.float32, rank, world)
        ret = np.zeros((cap, H), np.float32)
        for blk in back:
            off, n = int(blk[0, 0]), int(blk[0, 1])
            ret[off:off + n] = blk[1:1 + n]
    # 5. combine in pick order (y = 0; y += w_p * down_p), then the shared expert
    y = np.zeros((per_tok, H), np.float32)
    for t in range(per_tok):
        acc = np.zeros(H, np.float32)
        for p in range(K):
            acc = acc + np.float32(w[t, p]) * ret[sp.slot[t, p]]
        y[t] = acc + shared[t]
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "mailbox"])
@pytest.mark.parametrize("world", [2, 4])
def test_ep_decomposition_matches_single_rank(tmp_path, world, transport):
    """The whole EP forward on gloo ranks with the oracle's expert math, over
    both exchange layouts -- exactly the rows that exist (NCCL) and the fixed
    [source][cap] mailbox slots with empty slots and return offsets (NVLink) --
    against the single-rank oracle layer, bit for bit."""
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_ep_rank, args=(world, port, str(tmp_path), transport), nprocs=world, start_method="spawn",
                       join=True)
    wl, orc = workload(), oracle()
    lay, x_bits = wl.config_layer("c0")
    y_ref, _, _ = orc.moe_layer(orc.port(), lay, wl.bf16_bits_to_f32(x_bits))
    y_ep = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    assert np.array_equal(y_ep.view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_mailbox_exchange_returns_every_row_to_its_slot(world):
    """The NVLink exchange's addressing (receive slots with holes, return at
    the sender's offset): every pick's expert output lands in the sender's
    return buffer at that pick's send slot, for balanced and one-sided
    routing, and empty slots carry no expert."""
    rng = np.random.default_rng(world)
    E, K, T = 64, 4, 37
    per = E // world
    for skew in (False, True):
        plans, idxs = [], []
        for r in range(world):
            if skew:  # every pick on rank 0's experts
                idx = np.stack([rng.permutation(per)[:K] for _ in range(T)])
            else:
                idx = np.stack([rng.permutation(E)[:K] for _ in range(T)])
            idxs.append(idx)
            plans.append(plan.pack(idx, E, world))
        cap = T * K
        boxes = plan.mailbox_exchange(plans, cap)
        # owner p "computes" a row as (global expert, source rank, source slot) and returns it
        ret = [np.full((cap, 3), -1, np.int64) for _ in range(world)]
        for p, (expert, src_slot, offs) in enumerate(boxes):
            assert np.all((expert >= 0) == (src_slot >= 0))
            assert np.all(expert[expert >= 0] < per)
            for s in range(world):
                n = int((expert[s] >= 0).sum())
                assert np.all(expert[s, n:] == -1)  # rows first, then holes
                for j in range(n):
                    ret[s][offs[s] + j] = (p * per + expert[s, j], s, src_slot[s, j])
        for r in range(world):
            got = ret[r][plans[r].slot.ravel()]
            assert np.array_equal(got[:, 0], idxs[r].ravel())
            assert np.all(got[:, 1] == r)
            assert np.array_equal(got[:, 2], plans[r].slot.ravel())


def _setup_rank(rank: int, world: int, port: int, out_dir: str, case: str) -> None:
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)

    def exchange(rec):
        out = [None] * world
        dist.all_gather_object(out, rec)
        return out

    local = plan.NF_OK
    if case == "nomem" and rank == world - 1:
        local = plan.NF_ERR_NOMEM
    if case == "memset" and rank == 0:
        local = plan.NF_ERR_CUDA
    if case == "inner" and rank == 1:
        local = plan.NF_ERR_UNSUPPORTED  # its experts handle was refused before the communicator existed
    if case == "two" and rank in (1, 2):
        local = plan.NF_ERR_NOMEM if rank == 1 else plan.NF_ERR_CUDA
    mapped = not (case == "nomap" and rank == 1)
    st, what, n = plan.setup_agreement(exchange, local, True, True, lambda: mapped)
    # a last exchange after set-up: only reachable when every rank took the
    # same number of set-up exchanges (gloo would otherwise mismatch or hang)
    tail = exchange({"n": n})
    assert all(t["n"] == n for t in tail)
    np.save(os.path.join(out_dir, f"s{rank}.npy"), np.array([st, n], np.int64))
    with open(os.path.join(out_dir, f"s{rank}.txt"), "w") as f:
        f.write(what)
    dist.destroy_process_group()


@pytest.mark.parametrize("case,world", [("ok", 2), ("nomem", 2), ("memset", 4), ("nomap", 4), ("inner", 2),
                                        ("two", 4)])
def test_setup_agreement_every_rank_takes_the_same_exchanges(tmp_path, case, world):
    """A rank whose set-up fails -- its handle creation before the
    communicator existed, or its mailbox allocation or initialisation -- still
    joins the set-up exchange: every rank then returns that failure together,
    after the same number of exchanges (with several failing ranks, the lowest
    one's); a rank that cannot map a peer makes every rank fall back to NCCL
    together."""
    import torch.multiprocessing as mp

    mp.start_processes(_setup_rank, args=(world, _free_port(), str(tmp_path), case), nprocs=world,
                       start_method="spawn", join=True)
    res = [np.load(tmp_path / f"s{r}.npy") for r in range(world)]
    msgs = [(tmp_path / f"s{r}.txt").read_text() for r in range(world)]
    assert len({tuple(r) for r in res}) == 1 and len(set(msgs)) == 1  # every rank agrees
    st, n = int(res[0][0]), int(res[0][1])
    if case == "ok":
        assert (st, msgs[0], n) == (plan.NF_OK, "nvlink", 2)
    elif case == "nomem":
        assert st == plan.NF_ERR_NOMEM and f"rank {world - 1}" in msgs[0] and n == 1
    elif case == "memset":
        assert st == plan.NF_ERR_CUDA and "rank 0 (initialisation)" in msgs[0] and n == 1
    elif case == "inner":
        assert st == plan.NF_ERR_UNSUPPORTED and "rank 1 (handle creation)" in msgs[0] and n == 1
    elif case == "two":
        assert st == plan.NF_ERR_NOMEM and "rank 1 (device allocation)" in msgs[0] and n == 1
    else:
        assert (st, msgs[0], n) == (plan.NF_OK, "nccl", 3)
