"""Expert parallelism on 2 GPUs and on every GPU of the box (up to 8; one
process per GPU) against one GPU holding every expert: the layer outputs and
routes must be identical bit for bit, over both exchanges inside the library
-- NVLink peer memory (CUDA IPC mailboxes, run in graph mode for several
steps) and NCCL point-to-point, also with the hot experts replicated on
every rank (their picks computed where the token is).  Skipped on fewer
than two GPUs."""
import os
import socket
import sys

import numpy as np
import pytest

from helpers import REPO, nfm, workload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(case: str, world: int):
    """(layer, token bits of every rank)."""
    wl = workload()
    if case == "c1":
        lay, x = wl.config_layer("c1")
        return lay, np.array_split(x, world)
    if case == "uneven":  # all tokens on rank 0, none on rank 1
        lay, x = wl.config_layer("c1")
        return lay, [x] + [x[:0]] * (world - 1)
    # skewed (and skewed_rep, the same routing with experts 0-3 replicated):
    # Zipf log-prior on the bias sends most picks to the first experts (rank 0)
    cfg = dict(wl.CONFIGS["c1"])
    lay = wl.make_layer(cfg, seed=7)
    lay.bias = (lay.bias + np.log((np.arange(lay.experts) + 1.0) ** -1.1)).astype(np.float32)
    x = wl.make_tokens(cfg, seed=7, tokens=96 * world)
    return lay, np.array_split(x, world)


REPLICAS = [0, 1, 2, 3]  # the skewed routing's hottest experts


def _rank(rank: int, world: int, port: int, out_dir: str, case: str, transport: str) -> None:
    sys.path.insert(0, str(REPO / "tests"))
    os.environ["NF_EP_TRANSPORT"] = transport
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    m = nfm()
    gid = [m.ep_group_id() if rank == 0 else None]
    dist.broadcast_object_list(gid, src=0)
    lay, parts = _tokens(case, world)
    cap = max(p.shape[0] for p in parts)
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=max(cap, 1), device=rank, ep=(rank, world, gid[0]),
                       ep_replicas=REPLICAS if case == "skewed_rep" else None)
    layer.bind_layer(lay)
    got_transport = layer.ep_transport()
    xb = parts[rank]
    T = xb.shape[0]
    x = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).cuda() if T else torch.zeros((1, lay.hidden), dtype=torch.int16, device="cuda")
    y = torch.zeros((max(T, 1), lay.hidden), dtype=torch.float32, device="cuda")
    idx = torch.zeros((max(T, 1), lay.top_k), dtype=torch.int32, device="cuda")
    w = torch.zeros((max(T, 1), lay.top_k), dtype=torch.float32, device="cuda")
    for _ in range(2):  # two steps in a row reuse the buffers
        layer.forward(x, y, T, None, idx, w)
        layer.sync()
    first = y.cpu().numpy()[:T].copy()
    if got_transport == "nvlink":
        # graph replay on a dedicated stream: the epoch flags advance on the device
        layer.set_graph_mode(True)
        s = torch.cuda.Stream()
        y.zero_()
        torch.cuda.synchronize()
        for _ in range(4):
            layer.forward(x, y, T, None, idx, w, stream=s.cuda_stream)
        layer.sync(s.cuda_stream)
        assert np.array_equal(y.cpu().numpy()[:T].view(np.uint32), first.view(np.uint32))
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), y=first, idx=idx.cpu().numpy()[:T], w=w.cpu().numpy()[:T],
             transport=np.array(got_transport))
    dist.barrier()  # every rank's last forward is done before any handle of the group goes
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nvlink", "nccl"])
@pytest.mark.parametrize("case", ["c1", "uneven", "skewed", "skewed_rep"])
@pytest.mark.parametrize("ranks", ["two", "all"])
def test_ep_matches_one_gpu(tmp_path, case, transport, ranks):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2 if ranks == "two" else min(n, 8)
    if ranks == "all" and world == 2:
        pytest.skip("only two GPUs: covered by the two-rank case")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path), case, transport), nprocs=world,
                       start_method="spawn", join=True)
    m = nfm()
    lay, parts = _tokens(case, world)
    xb = np.concatenate(parts)
    T = xb.shape[0]
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    x = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).cuda()
    y = torch.zeros((T, lay.hidden), dtype=torch.float32, device="cuda")
    idx = torch.zeros((T, lay.top_k), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, lay.top_k), dtype=torch.float32, device="cuda")
    layer.forward(x, y, T, None, idx, w)
    layer.sync()
    got = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    assert all(str(g["transport"]) == transport for g in got), [str(g["transport"]) for g in got]
    y_ep = np.concatenate([g["y"] for g in got])
    assert np.array_equal(np.concatenate([g["idx"] for g in got]), idx.cpu().numpy())
    assert np.array_equal(np.concatenate([g["w"] for g in got]).view(np.uint32), w.cpu().numpy().view(np.uint32))
    assert np.array_equal(y_ep.view(np.uint32), y.cpu().numpy().view(np.uint32))
    layer.close()


def _skip_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    """Step 1: both ranks forward.  Step 2: rank 1 skips its forward (decided
    on the host); rank 0's bounded flag waits run out and its sync reports
    the timeout.  Then both ranks drop the group and make a new one, whose
    forward must again equal one GPU's."""
    sys.path.insert(0, str(REPO / "tests"))
    os.environ["NF_EP_TRANSPORT"] = "nvlink"
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    m = nfm()
    lay, parts = _tokens("c1", world)
    cap = max(p.shape[0] for p in parts)

    def group():
        gid = [m.ep_group_id() if rank == 0 else None]
        dist.broadcast_object_list(gid, src=0)
        layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                           swiglu_limit=lay.swiglu_limit, max_tokens=cap, device=rank, ep=(rank, world, gid[0]))
        layer.bind_layer(lay)
        return layer

    xb = parts[rank]
    T = xb.shape[0]
    x = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).cuda()
    y = torch.zeros((T, lay.hidden), dtype=torch.float32, device="cuda")
    layer = group()
    assert layer.ep_transport() == "nvlink"
    layer.forward(x, y, T)
    layer.sync()
    dist.barrier()
    status = "none"
    if rank == 0:
        layer.forward(x, y, T)  # rank 1 never sends: the waits give up after their budget
        try:
            layer.sync()
            status = "ok"
        except m.NfError as e:
            status = m.NF_ERR.get(e.status, str(e.status))
    dist.barrier()  # rank 0's forward (with its given-up waits) is complete before the group goes
    layer.close()
    dist.barrier()
    layer = group()
    y.zero_()
    layer.forward(x, y, T)
    layer.sync()
    np.savez(os.path.join(out_dir, f"s{rank}.npz"), y=y.cpu().numpy(), status=np.array(status))
    dist.barrier()
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def test_ep_rank_that_skips_a_step_times_out_and_the_group_recovers(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects for a test where a rank drops out
    world = 2
    mp.start_processes(_skip_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    got = [np.load(tmp_path / f"s{r}.npz") for r in range(world)]
    assert str(got[0]["status"]) == "TIMEOUT", str(got[0]["status"])
    m = nfm()
    lay, parts = _tokens("c1", world)
    xb = np.concatenate(parts)
    T = xb.shape[0]
    layer = m.MoeLayer(lay.hidden, lay.experts, lay.top_k, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    x = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).cuda()
    y = torch.zeros((T, lay.hidden), dtype=torch.float32, device="cuda")
    layer.forward(x, y, T)
    layer.sync()
    y_ep = np.concatenate([g["y"] for g in got])
    assert np.array_equal(y_ep.view(np.uint32), y.cpu().numpy().view(np.uint32))
    layer.close()
