#!/usr/bin/env python
"""Benchmark of the B200 NVFP4 MoE layer (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (N = 1): the benchmark's configs[1], the decode batch --
H2048, 64 routed experts top-4 (scale 2.5), expert intermediate 1536, one
BF16 shared expert of 1536, 64 tokens -- with seeded synthetic weights and
activations.  A step is one forward of the layer over the 64 tokens, inputs
resident in HBM (the 340 MB of weights exceed the 126 MB L2, so no flush is
needed between steps).  `value` is tokens/s of the whole job; the line also
carries us/layer, the per-stage device times, the HBM roofline of the
dominant kernel (the grouped gate/up GEMM), the end-to-end number through
the host-buffer C-ABI call, the reference CPU path timed on this host, and a
secondary prefill measurement (configs[2], 8192 tokens, tensor roofline) and
the dense NVFP4 MLP of configs[4] (decode and prefill batches).

With N > 1 (torchrun), the layer is expert-parallel: each rank owns E/N
experts and brings its own 64-token decode batch (weak scaling: tokens per
GPU fixed); rows travel to the experts' owners and back inside the library,
over NVLink peer memory (NCCL point-to-point when the ranks cannot map each
other's buffers; config.ep_transport says which).  value sums the tokens of
all ranks over the max-over-ranks device time.

Each rank of an expert-parallel run also checks its EP outputs (y, routes)
bit for bit against a single-GPU handle holding every expert on the same
tokens and reports the verdict as "ep_parity".

--impl reference times the reference's own CPU implementation (its sources
compiled under oracle/_ref, else the C restatement) on this host's cores over
the same workload: each step is the full 64-token decode batch.  Under
torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path


def cpu_threads() -> int:
    """Host threads this process may run on (its CPU affinity set)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


# The CPU legs use every host core the process may run on.  torchrun exports
# OMP_NUM_THREADS=1 to each rank, so this overrides rather than defaults; the
# oracle's OpenMP runtime reads it when the oracle library loads.
os.environ["OMP_NUM_THREADS"] = str(cpu_threads())

import numpy as np  # noqa: E402

REPO = Path(__file__).resolve().parent
PKG = REPO / "ninfer_nvfp4_glm-5.3_flash_2x_dgxspark_b200"


def load_module(name: str, path: Path):
    """Imports a module by file path (the package folder's name is not a
    Python identifier)."""
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


wl = load_module("nf_workload", PKG / "workload.py")

METRIC = "MoE layer tokens/s (decode c1, T=64) + % HBM BW; prefill c2 tokens/s + % NVFP4 TC peak"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks() -> tuple[float, float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout_s: float = 5.0) -> None:
        """Returns once nvidia-smi has printed its first sample (it takes a
        few hundred ms to start), so the loop that follows is sampled."""
        t0 = time.monotonic()
        while self.proc is not None and not self.lines and time.monotonic() - t0 < timeout_s:
            if self.proc.poll() is not None:
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def steps_for(step, stream, seconds: float, dist, torch) -> int:
    """Steps that take about `seconds` (from 20 timed steps), the same number
    on every rank: the largest rank's count wins."""
    n0 = 20
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(n0):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    per_ms = max(ev0.elapsed_time(ev1) / n0, 1e-3)
    n = int(min(200000, max(100, math.ceil(seconds * 1e3 / per_ms))))
    if dist:
        t = torch.tensor([n], device="cuda", dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = int(t.item())
    return n


def merge_clocks(per_rank: list) -> dict:
    """Rank 0's clock record plus every rank's median SM clock and the union
    of the throttle reasons any rank saw."""
    out = dict(per_rank[0])
    out["reasons"] = sorted({r for c in per_rank for r in (c.get("reasons") or [])})
    out["per_rank_sm_mhz"] = [c.get("sm_mhz") for c in per_rank]
    out["per_rank_samples"] = [c.get("samples") for c in per_rank]
    return out


def ep_parity_check(m, torch, lay, x, T: int, device: int, y_ep, idx_ep, w_ep) -> bool:
    """True when the expert-parallel outputs of this rank's tokens (y, route
    indices and weights) equal bit for bit those of a single-GPU handle that
    holds every expert, run on the same tokens on this rank's GPU."""
    H, K = lay.hidden, lay.top_k
    ref = m.MoeLayer(H, lay.experts, K, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                     swiglu_limit=lay.swiglu_limit, max_tokens=max(T, 1), device=device)
    ref.bind_layer(lay)
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    ref.forward(x, y, T, None, idx, w)
    ref.sync()
    ok = (np.array_equal(y.cpu().numpy().view(np.uint32), np.asarray(y_ep).view(np.uint32))
          and np.array_equal(idx.cpu().numpy(), np.asarray(idx_ep))
          and np.array_equal(w.cpu().numpy().view(np.uint32), np.asarray(w_ep).view(np.uint32)))
    ref.close()
    return bool(ok)


def decode_bytes(lay, active: int, tokens: int) -> dict:
    """Algorithmic HBM bytes of one decode step and of the gate/up kernel."""
    H, I, Is, E = lay.hidden, lay.inter, lay.shared_inter, lay.experts
    gu_w = active * (2 * I * H // 2 + 2 * I * H // 16)
    dn_w = active * (H * I // 2 + H * I // 16)
    pairs = tokens * lay.top_k
    act_gu = pairs * (H // 2 + H // 16)      # quantised dispatch rows read
    h_out = pairs * (I // 2 + I // 16)       # down-input codes written
    shared = 3 * Is * H * 2
    router = E * H * 2 + E * 4
    io = tokens * H * 2 + tokens * H * 4     # x in, y out
    return {"gate_up": gu_w + act_gu + h_out, "layer": gu_w + dn_w + shared + router + io}


def ep_rank_bytes(lay, idx_all: list, rank: int, world: int) -> dict:
    """Algorithmic HBM bytes one rank of an expert-parallel decode step moves.

    idx_all[r] holds rank r's routes [T_r, k].  Rank `rank` streams the
    weights of the experts it owns that received at least one row from any
    rank, the replicated shared expert and router, its own tokens' input and
    output rows, and the exchanged rows: every row it receives is written
    into its mailbox and read by the dispatch (BF16, 2H B each way), and
    every down row it computes is written back to the source and read by the
    source's combine (BF16, 2H B each way).  The gate/up figure is the same
    kernel's share as in decode_bytes, over the rows this rank received."""
    H, I, Is, E, k = lay.hidden, lay.inter, lay.shared_inter, lay.experts, lay.top_k
    local = E // world
    lo, hi = rank * local, (rank + 1) * local
    picks = np.concatenate([np.asarray(a).ravel() for a in idx_all]) if idx_all else np.zeros(0, np.int64)
    mine = picks[(picks >= lo) & (picks < hi)]
    active = int(np.unique(mine).size)
    recv = int(mine.size)
    T = int(np.asarray(idx_all[rank]).shape[0])
    gu_w = active * (2 * I * H // 2 + 2 * I * H // 16)
    dn_w = active * (H * I // 2 + H * I // 16)
    act_gu = recv * (H // 2 + H // 16)
    h_out = recv * (I // 2 + I // 16)
    exchange = recv * H * 2 * 2 + recv * H * 2 * 2
    # the single-GPU layer figure's terms (weights, shared expert, router, x in
    # and y out) plus the exchange
    layer = gu_w + dn_w + 3 * Is * H * 2 + E * H * 2 + E * 4 + T * H * 2 + T * H * 4 + exchange
    return {"gate_up": gu_w + act_gu + h_out, "layer": layer, "active_owned": active, "rows_received": recv,
            "tokens": T}


def prefill_flops(lay, tokens: int) -> dict:
    H, I, Is, E, k = lay.hidden, lay.inter, lay.shared_inter, lay.experts, lay.top_k
    return {"fp4": tokens * k * (2 * H * 2 * I + 2 * I * H), "fp4_gate_up": tokens * k * 2 * H * 2 * I,
            "bf16_shared": tokens * 3 * 2 * Is * H, "router": 2 * tokens * E * H}


def cpu_reference_rate(lay, x_bits, tokens: int) -> tuple[float, dict]:
    """Tokens/s of the reference CPU path on `tokens` tokens of the batch."""
    orc = load_module("nf_oracle_py", REPO / "oracle" / "oracle.py")
    lib = orc.ref()
    kind = "reference"
    if lib is None:
        lib, kind = orc.port(), "port"
    x = wl.bf16_bits_to_f32(x_bits[:tokens])
    t0 = time.perf_counter()
    orc.moe_layer(lib, lay, x)
    dt = time.perf_counter() - t0
    info = {"kind": kind, "cores": int(os.environ["OMP_NUM_THREADS"]),
            "sample": f"{tokens} of the {x_bits.shape[0]} decode tokens, one token at a time with OpenMP GEMV rows "
                      "(the reference's own schedule)"}
    return tokens / dt, info


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU path on the same workload as our arm's headline:
    each step is the whole 64-token decode batch, on every host thread."""
    if rank != 0:
        return
    lay, x_bits = wl.config_layer("c1")
    T = x_bits.shape[0]
    for _ in range(args.warmup):
        cpu_reference_rate(lay, x_bits, T)
    info = {}
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, info = cpu_reference_rate(lay, x_bits, T)
    total = time.perf_counter() - t0
    value = T * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (NVFP4 fake-quant)",
        "data": "synthetic",
        "config": {"workload": "c1 decode: H2048 E64 k4 I1536 Is1536 T64 scale2.5 (configs[1])", "tokens_per_step": T,
                   "omp_num_threads": int(os.environ["OMP_NUM_THREADS"])},
        "cpu_baseline": {"value": value, "unit": "tokens/s", **info},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local: int) -> None:
    import torch

    m = load_module("nf_moe", PKG / "nf_moe.py")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    hbm_peak, bf16_peak, peak_src = peaks()
    fp4_peak = 4 * bf16_peak  # dense FP4 is 4x dense BF16 on this part

    lay, x_bits = wl.config_layer("c1")
    if world > 1:
        # every rank brings its own decode batch of the same size
        x_bits = wl.make_tokens(wl.CONFIGS["c1"], seed=1 + rank)
    T, H, K = x_bits.shape[0], lay.hidden, lay.top_k
    ep = None
    if world > 1:
        # expert parallel: this rank owns E / world experts; the group id
        # comes from rank 0
        gid = [m.ep_group_id() if rank == 0 else None]
        dist.broadcast_object_list(gid, src=0)
        ep = (rank, world, gid[0])
    layer = m.MoeLayer(H, lay.experts, K, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T, device=local, ep=ep)
    layer.bind_layer(lay)
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    # The layer runs on its own stream; with graph mode on, the first forward
    # for a token count captures the layer's launches into a CUDA graph and
    # later forwards replay it (one launch per step on the host side).
    # (Expert-parallel forwards over NVLink peer memory run in graph mode
    # too; over the NCCL fallback they synchronise the host once for the row
    # counts and the library launches them directly.)
    tstream = torch.cuda.Stream()
    stream = tstream.cuda_stream
    layer.set_graph_mode(True)

    def step():
        layer.forward(x, y, T, None, idx, w, stream=stream)

    for _ in range(args.warmup):
        step()
    layer.sync(stream)
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first()
    # settle clocks under the same load before timing, ~1 s; every rank of an
    # expert-parallel group takes the same number of steps (steps_for agrees
    # on it), since each forward exchanges rows with every other rank
    n_settle = steps_for(step, tstream, 1.0, dist, torch)
    for _ in range(n_settle):
        step()
    tstream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(tstream)
    for _ in range(args.steps):
        step()
    ev1.record(tstream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    # Stage times: the same K steps again, launched directly (profiling
    # bypasses the graph) with events around each kernel on its stream.
    layer.profile(True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    stages, nfw = layer.stage_times()
    layer.profile(False)
    for _ in range(max(1, n_settle // 2)):
        step()
    tstream.synchronize()
    clk = clocks.stop()
    layer.sync(stream)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        per_rank_clk = [None] * world
        dist.all_gather_object(per_rank_clk, clk)
        clk = merge_clocks(per_rank_clk)
        dist.barrier()
    stage_ms = {k: v / max(nfw, 1) for k, v in stages.items()}
    idx_h = idx.cpu().numpy()
    y_ep = y.cpu().numpy()
    w_ep = w.cpu().numpy()
    if dist:
        idx_all = [None] * world
        dist.all_gather_object(idx_all, idx_h)
        mine = ep_rank_bytes(lay, idx_all, rank, world)
        all_bytes = [ep_rank_bytes(lay, idx_all, r, world) for r in range(world)]
        active = int(np.unique(np.concatenate([a.ravel() for a in idx_all])).size)
        nbytes = {"gate_up": mine["gate_up"], "layer": sum(b["layer"] for b in all_bytes)}
    else:
        active = int(np.unique(idx_h).size)
        nbytes = decode_bytes(lay, active, T)
        mine = None

    # expert-parallel outputs against one GPU holding every expert, bit for bit
    ep_ok = None
    if dist:
        ep_ok = ep_parity_check(m, torch, lay, x, T, local, y_ep, idx_h, w_ep)
        flag = torch.tensor([1 if ep_ok else 0], device="cuda", dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ep_ok = bool(flag.item())

    # end to end through the host-buffer C-ABI call (pinned host memory)
    xh = torch.from_numpy(wl.bf16_bits_to_f32(x_bits)).pin_memory().numpy()
    outs = (torch.empty((T, H), dtype=torch.float32).pin_memory().numpy(),
            torch.empty((T, K), dtype=torch.int32).pin_memory().numpy(),
            torch.empty((T, K), dtype=torch.float32).pin_memory().numpy())
    for _ in range(args.warmup):
        layer.forward_host(xh, out=outs)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer.forward_host(xh, out=outs)
    e2e_s = (time.perf_counter() - t0) / args.steps
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    line = None
    if rank == 0:
        gu_ms = stage_ms["gate_up"]
        achieved = nbytes["gate_up"] / (gu_ms * 1e-3) / 1e9
        # DRAM read + write of one gate/up launch from the committed ncu summary
        traffic = None
        tf = REPO / "profiles" / "gemm_gate_up_c1_decode.md"
        if tf.exists() and world == 1:
            for ln in tf.read_text().splitlines():
                if ln.startswith("traffic_bytes_per_launch:"):
                    traffic = int(ln.split(":")[1])
        # fused router, permutation, dispatch, gate/up GEMM, down GEMM,
        # combine; + shared gate/up and down GEMMs on the side stream
        launches_per_step = 8 if lay.shared_inter > 0 else 6
        if world > 1:
            # + pack, send, receive wait, return, return wait (NVLink) or
            # + pack and two row gathers (NCCL, whose own kernels are not counted)
            launches_per_step += 4 if layer.ep_transport() == "nvlink" else 3
        layer_gbs = nbytes["layer"] / (ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "grouped NVFP4 gate/up GEMM (SwiGLU + quant fused)",
                "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                "peak_source": peak_src, "traffic": traffic,
                "algorithmic_bytes_per_launch": nbytes["gate_up"],
                "layer_achieved_gbs": layer_gbs, "layer_frac": layer_gbs / (world * hbm_peak),
                "layer_algorithmic_bytes": nbytes["layer"]}
        if world > 1:
            roof["per_rank"] = ("achieved/frac: rank 0's gate/up bytes (its owned experts with rows, the rows it "
                                "received) over rank 0's gate/up time; layer_frac: every rank's bytes over "
                                "world x the max-over-ranks step time x peak")
            roof["rank0"] = mine
        line = {
            "metric": METRIC, "value": world * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "nvfp4 (E2M1 x UE4M3/16, fp32 accumulate); bf16 shared expert", "data": "synthetic",
            "config": {"workload": "c1 decode: H2048 E64 k4 I1536 Is1536 T64 scale2.5 (configs[1])",
                       "tokens_per_gpu": T, "parallelism": f"ep{world}" if world > 1 else "single",
                       "ep_transport": layer.ep_transport(),
                       "l2": "no flush: the 340 MB of weights streamed per step exceed the 126 MB L2",
                       "active_experts": active},
            "stages_us": {k: 1e3 * v for k, v in stage_ms.items()},
            "timing": "timed steps replay a CUDA graph on a dedicated stream; stages_us from K more steps "
                      "launched directly with events around each kernel",
            "roofline": roof,
            "e2e": {"value": world * T / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4 + T * K * 8, "ms_per_step": 1e3 * e2e_s},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if ep_ok is not None:
            line["ep_parity"] = ep_ok
            line["ep_parity_check"] = ("every rank's y, routes and route weights equal bit for bit those of a "
                                       "single-GPU handle holding all experts on the same tokens")
    if world == 1 and not args.no_prefill:
        line["prefill"] = run_prefill(args, m, torch, fp4_peak, bf16_peak, peak_src)
        line["dense"] = run_dense(args, m, torch, hbm_peak, fp4_peak, peak_src)
        if not args.no_stack:
            line["stack_c4"] = run_stack(args, m, torch, hbm_peak)
    if not args.no_prefill:
        tph = run_tp_head(args, m, torch, rank, world, local, dist, hbm_peak)
        if rank == 0:
            line["tp_lm_head"] = tph
    if not args.no_prefill:
        ep3 = run_ep_c3(args, m, torch, rank, world, local, dist)
        ep3c = run_ep_c3(args, m, torch, rank, world, local, dist, lam=wl.C3_LAMBDA_CALIBRATED)
        if rank == 0:
            line["ep_c3"] = ep3
            line["ep_c3_calibrated"] = ep3c
    if rank == 0 and world == 1:
        rate, info = cpu_reference_rate(lay, x_bits, T)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", **info}
    layer.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args, m, torch, fp4_peak, bf16_peak, peak_src) -> dict:
    lay, x_bits = wl.config_layer("c2")
    T, H, K = x_bits.shape[0], lay.hidden, lay.top_k
    layer = m.MoeLayer(H, lay.experts, K, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    layer.set_expert_gemm(args.expert_gemm)
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        layer.forward(x, y, T, None, idx, w, stream=stream)
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 20))
    # the step time unprofiled (the kernels hand rows over and overlap as in
    # service); then the per-stage split from as many profiled steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        layer.forward(x, y, T, None, idx, w, stream=stream)
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    layer.profile(True)
    for _ in range(steps):
        layer.forward(x, y, T, None, idx, w, stream=stream)
    torch.cuda.synchronize()
    stages, nfw = layer.stage_times()
    layer.profile(False)
    layer.sync(stream)
    counts = np.bincount(idx.cpu().numpy().ravel(), minlength=lay.experts)
    # the screened router's candidates per token (-1: every chain)
    cand = layer.debug_read("screen_count", np.int32, T)
    fl = prefill_flops(lay, T)
    gu_ms = stages["gate_up"] / max(nfw, 1)
    dn_ms = stages["down"] / max(nfw, 1)
    t_ideal = fl["fp4"] / (fp4_peak * 1e12) + (fl["bf16_shared"] + fl["router"]) / (bf16_peak * 1e12)
    layer.close()
    return {
        "workload": "c2 prefill: c1 shapes, T8192, bias tuned to 512 +- 10% tokens per expert (configs[2])",
        "tokens_per_s": T / (ms * 1e-3), "ms_per_step": ms, "steps": steps,
        "stages_us": {k: 1e3 * v / max(nfw, 1) for k, v in stages.items()},
        "timing": "ms_per_step over K unprofiled steps (direct launches, stages overlapping as in service); "
                  "stages_us from K more steps with an event around each kernel (kernels kept apart)",
        "expert_gemms": {"one_sm": "one SM per 128 x 256 tile, 256-K stages", "wide": "one SM, 512-K stages",
                         "pair": "CTA pairs (cta_group::2), 256 x 256 tiles, A resident"}[args.expert_gemm],
        "expert_tokens_min_max": [int(counts.min()), int(counts.max())],
        "router_screen": {"mean_candidates": float(np.mean(np.where(cand < 0, lay.experts, cand))),
                          "all_chain_tokens": int(np.sum(cand < 0)), "exact_chains": int(np.sum(np.where(cand < 0, lay.experts, cand)))},
        "fp4_tflops_layer": fl["fp4"] / (ms * 1e-3) / 1e12,
        "fp4_frac_layer": fl["fp4"] / (ms * 1e-3) / 1e12 / fp4_peak,
        "mixed_roofline_frac": t_ideal / (ms * 1e-3),
        "roofline": {"bound": "tensor", "kernel": "grouped NVFP4 gate/up GEMM",
                     "achieved": fl["fp4_gate_up"] / (gu_ms * 1e-3) / 1e12, "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": fl["fp4_gate_up"] / (gu_ms * 1e-3) / 1e12 / fp4_peak,
                     "peak_source": f"4 x {peak_src} dense BF16 ({bf16_peak:.0f} TFLOP/s); nominal dense FP4 9000",
                     "down_tflops": (fl["fp4"] - fl["fp4_gate_up"]) / (dn_ms * 1e-3) / 1e12},
    }


def choose_replicas(counts_src: np.ndarray, e_per_rank: int, max_rep: int = 16) -> list[int]:
    """Hot experts to replicate on every rank, greedily: counts_src[r, e] are
    the picks of expert e made by rank r's tokens; with replica set R rank r
    computes its own picks of R and every rank's picks of the experts it owns
    outside R.  Adds experts in descending pick count while that lowers the
    busiest rank's load by 2% or more."""
    world, E = counts_src.shape
    tot = counts_src.sum(0)

    def busiest(rs):
        load = np.zeros(world)
        for e in range(E):
            if e in rs:
                load += counts_src[:, e]
            else:
                load[e // e_per_rank] += tot[e]
        return load.max()

    reps, best = set(), busiest(set())
    for e in np.argsort(-tot, kind="stable")[:max_rep]:
        b = busiest(reps | {int(e)})
        if b < 0.98 * best:
            reps, best = reps | {int(e)}, b
    return sorted(reps)


def run_ep_c3(args, m, torch, rank: int, world: int, local: int, dist, lam: float = 1.0) -> dict:
    """16384 tokens per step split over the ranks (strong scaling),
    experts sharded evenly, router bias + lam * Zipf(1.1) log-prior (at the
    configuration's literal lam = 1 nearly every pick lands on the first
    experts, i.e. on rank 0; at the calibrated lam the pick shares follow the
    Zipf distribution most closely).  Device time per step, max over ranks.
    With more than one rank the step is timed twice: experts only sharded,
    then with the hot experts replicated on every rank (choose_replicas over
    the first run's picks; the product path's number)."""
    first = _run_ep_c3_once(args, m, torch, rank, world, local, dist, lam, None)
    if world == 1:
        return first
    e_per_rank = first["experts"] // world
    counts = np.zeros((world, first["experts"]), dtype=np.int64)
    counts[rank] = np.bincount(first["idx"].ravel(), minlength=first["experts"])
    t = torch.from_numpy(counts).cuda()
    dist.all_reduce(t)
    counts = t.cpu().numpy()
    reps = choose_replicas(counts, e_per_rank)
    out = _run_ep_c3_once(args, m, torch, rank, world, local, dist, lam, reps)
    out["replicas"] = reps
    out["ms_per_step_experts_sharded_only"] = first["ms_per_step"]
    out["ep_parity_experts_sharded_only"] = first.get("ep_parity")
    # picks each rank computes, with and without the replicas
    tot = counts.sum(0)
    for key, rs in (("picks_by_computing_rank_sharded_only", set()), ("picks_by_computing_rank", set(reps))):
        load = np.zeros(world, dtype=np.int64)
        for e in range(counts.shape[1]):
            if e in rs:
                load += counts[:, e]
            else:
                load[e // e_per_rank] += tot[e]
        out[key] = [int(v) for v in load]
    return out


def _run_ep_c3_once(args, m, torch, rank: int, world: int, local: int, dist, lam: float, replicas) -> dict:
    lay, x_all = wl.config_layer("c3", zipf_lambda=lam)
    T_all, H, K = x_all.shape[0], lay.hidden, lay.top_k
    per = T_all // world
    xb = x_all[rank * per:(rank + 1) * per]
    ep = None
    if world > 1:
        gid = [m.ep_group_id() if rank == 0 else None]
        dist.broadcast_object_list(gid, src=0)
        ep = (rank, world, gid[0])
    layer = m.MoeLayer(H, lay.experts, K, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=per, device=local, ep=ep, ep_replicas=replicas)
    layer.bind_layer(lay)
    x = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).cuda()
    y = torch.empty((per, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((per, K), dtype=torch.int32, device="cuda")
    w = torch.empty((per, K), dtype=torch.float32, device="cuda")
    ts = torch.cuda.Stream()
    steps = max(3, min(args.steps, 10))
    for _ in range(args.warmup):
        layer.forward(x, y, per, None, idx, w, stream=ts.cuda_stream)
    ts.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(ts)
    for _ in range(steps):
        layer.forward(x, y, per, None, idx, w, stream=ts.cuda_stream)
    ev1.record(ts)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    layer.sync(ts.cuda_stream)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    idx_h = idx.cpu().numpy()
    # where this rank's picks are computed: the expert's owner, or this rank
    # for a replicated expert
    dest = idx_h.ravel() // (lay.experts // world)
    if replicas:
        dest = np.where(np.isin(idx_h.ravel(), replicas), rank, dest)
    owners = np.bincount(dest, minlength=world)
    out = {"workload": f"c3: c1 shapes, 16384 tokens per step split over the ranks, Zipf(1.1) log-prior "
                       f"lambda = {lam:g} (configs[3])", "tokens_per_s": T_all / (ms * 1e-3), "ms_per_step": ms,
           "steps": steps,
           "scaling": "strong", "parallelism": f"ep{world}" if world > 1 else "single",
           "rank0_picks_by_owner": [int(c) for c in owners],
           # rank 0's (token, pick) rows that cross to another rank: dispatched
           # as BF16 rows (H * 2 B) and returned as BF16 down rows (H * 2 B)
           "rank0_remote_bytes": {"dispatch": int(owners.sum() - owners[0]) * H * 2,
                                  "combine": int(owners.sum() - owners[0]) * H * 2}}
    if dist:
        ok = ep_parity_check(m, torch, lay, x, per, local, y.cpu().numpy(), idx_h, w.cpu().numpy())
        flag = torch.tensor([1 if ok else 0], device="cuda", dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        out["ep_parity"] = bool(flag.item())
        dist.barrier()  # every rank's last forward is done before any handle of the group goes
    layer.close()
    if world > 1 and replicas is None:
        out["idx"], out["experts"] = idx_h, lay.experts
    return out


def run_dense(args, m, torch, hbm_peak, fp4_peak, peak_src) -> dict:
    """configs[4]'s dense NVFP4 MLP (layers 0-2: H2048, I10240) at the decode
    batch (64 tokens; HBM roofline: every weight byte once per step) and at a
    prefill batch (8192 tokens; FP4 tensor roofline).  Decode steps replay a
    CUDA graph on a dedicated stream; the 35 MB of weights fit in L2, so each
    timed decode step is preceded by an L2 flush (a 256 MB write, outside the
    per-step events)."""
    cfg = wl.DENSE_CONFIGS["c4_dense"]
    H, I = cfg["hidden"], cfg["inter"]
    lay = wl.make_dense_layer(H, I, seed=4)
    out = {"workload": "c4 dense NVFP4 MLP (layers 0-2): H2048 I10240, swiglu_clamp_bf16 (configs[4])"}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for T in (64, 8192):
        mlp = m.DenseMlp(H, I, swiglu_limit=lay.swiglu_limit, max_tokens=T)
        mlp.bind_layer(lay)
        x = torch.from_numpy(wl.make_tokens(dict(hidden=H, tokens=T), 4).view(np.int16)).cuda()
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        ts = torch.cuda.Stream()
        mlp.set_graph_mode(True)
        for _ in range(args.warmup):
            mlp.forward(x, y, T, stream=ts.cuda_stream)
        ts.synchronize()
        steps = max(3, min(args.steps, 20))
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            with torch.cuda.stream(ts):
                flush.fill_(1)
            e0.record(ts)
            mlp.forward(x, y, T, stream=ts.cuda_stream)
            e1.record(ts)
        ts.synchronize()
        ms = float(np.mean([e0.elapsed_time(e1) for e0, e1 in evs]))
        mlp.profile(True)
        for _ in range(steps):
            with torch.cuda.stream(ts):
                flush.fill_(1)
            mlp.forward(x, y, T, stream=ts.cuda_stream)
        ts.synchronize()
        stages, nfw = mlp.stage_times()
        mlp.profile(False)
        mlp.sync(ts.cuda_stream)
        mlp.close()
        st_us = {k: 1e3 * v / max(nfw, 1) for k in ("permute", "gate_up", "down", "combine") for v in [stages[k]]}
        if T == 64:
            nbytes = lay.weight_bytes() + T * H * 2 + T * H * 4
            gb = nbytes / (ms * 1e-3) / 1e9
            out["decode"] = {"tokens": T, "us_per_layer": 1e3 * ms, "tokens_per_s": T / (ms * 1e-3),
                             "stages_us": st_us, "algorithmic_bytes": nbytes, "achieved_gbs": gb,
                             "hbm_frac": gb / hbm_peak, "peak_source": peak_src}
        else:
            flops = T * 3 * 2 * H * I
            tf = flops / (ms * 1e-3) / 1e12
            gu_tf = T * 2 * H * 2 * I / (st_us["gate_up"] * 1e-6) / 1e12
            out["prefill"] = {"tokens": T, "us_per_layer": 1e3 * ms, "tokens_per_s": T / (ms * 1e-3),
                              "stages_us": st_us, "fp4_tflops": tf, "fp4_frac": tf / fp4_peak,
                              "gate_up_fp4_frac": gu_tf / fp4_peak,
                              "peak_source": f"4 x {peak_src} dense BF16"}
    del flush
    return out


def run_tp_head(args, m, torch, rank: int, world: int, local: int, dist, hbm_peak: float) -> dict:
    """The lm_head of configs[4] ([151552, 2048] BF16) through the tensor-
    parallel linear (exact gemv_bf16 rows, gathered on every rank) and the
    greedy pick, at the stack's batch sizes.  HBM roofline per rank: its
    row block's weight bytes once per call."""
    rows, cols = wl.STACK_CONFIGS["c4"]["vocab"], wl.STACK_CONFIGS["c4"]["hidden"]
    gid = None
    if world > 1:
        g = [m.ep_group_id() if rank == 0 else None]
        dist.broadcast_object_list(g, src=0)
        gid = g[0]
    tp = m.TpGroup(max_tokens=max(wl.STACK_BATCHES), max_rows=rows, rank=rank, world=world, group_id=gid,
                   device=local)
    r0, r1 = tp.split(rows)
    rng = np.random.default_rng(40)
    w = torch.from_numpy(wl.f32_to_bf16_bits(rng.standard_normal((r1 - r0, cols), dtype=np.float32)
                                             * np.float32(0.02)).view(np.int16)).cuda()
    ts = torch.cuda.Stream()
    out = {"workload": "configs[4] lm_head [151552, 2048] BF16: exact row-split GEMV + NVLink gather + greedy pick",
           "transport": tp.transport(), "per_batch": {}}
    for T in wl.STACK_BATCHES:
        x = torch.from_numpy(rng.standard_normal((T, cols), dtype=np.float32)).cuda()
        idx = torch.empty(T, dtype=torch.int32, device="cuda")
        for _ in range(args.warmup):
            tp.linear_bf16(w, rows, cols, x, T, None, stream=ts.cuda_stream)
            tp.argmax(T, rows, idx, stream=ts.cuda_stream)
        tp.sync(ts.cuda_stream)
        steps = max(3, min(args.steps, 20 if T <= 16 else 5))
        if dist:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(ts)
        for _ in range(steps):
            tp.linear_bf16(w, rows, cols, x, T, None, stream=ts.cuda_stream)
            tp.argmax(T, rows, idx, stream=ts.cuda_stream)
        ev1.record(ts)
        tp.sync(ts.cuda_stream)
        ms = ev0.elapsed_time(ev1) / steps
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        gbs = (r1 - r0) * cols * 2 / (ms * 1e-3) / 1e9
        out["per_batch"][str(T)] = {"us": 1e3 * ms, "tokens_per_s": T / (ms * 1e-3), "rank_weight_gbs": gbs,
                                    "hbm_frac": gbs / hbm_peak}
    if dist:
        dist.barrier()  # every rank's last call is done before any handle of the group goes
    tp.close()
    return out


def run_stack(args, m, torch, hbm_peak: float) -> dict:
    """the full synthetic decoder stack (46 layers: 3 dense NVFP4
    MLPs, 42 NVFP4 MoE layers of c1's shapes, 1 BF16-expert MoE layer; BF16
    GQA 32/4/128 attention; vocab 151552), greedy decode with a 2048-token
    context (caches filled on the device with a pseudo-random history) at
    batch 1/16/64/256 on one GPU.  A step is one token for every sequence;
    timed as CUDA-graph replays of the whole step."""
    cfg = dict(wl.STACK_CONFIGS["c4"])
    layers = getattr(args, "stack_layers", None)
    if layers and layers != cfg["layers"]:
        # a shorter stack of the same shapes (profiling): one dense, one BF16-expert layer
        cfg.update(layers=layers, dense_layers=1, bf16_expert_layers=1)
    batches = tuple(getattr(args, "stack_batches", None) or wl.STACK_BATCHES)
    t0 = time.perf_counter()
    model = wl.make_stack(cfg, seed=4, share=True)
    st = m.DecoderStack(vocab=cfg["vocab"], hidden=cfg["hidden"], layers=cfg["layers"],
                        dense_layers=cfg["dense_layers"], bf16_expert_layers=cfg["bf16_expert_layers"],
                        dense_inter=cfg["dense_inter"], experts=cfg["experts"], top_k=cfg["top_k"], inter=cfg["inter"],
                        shared_inter=cfg["shared_inter"], routed_scaling=cfg["scaling"], q_heads=cfg["q_heads"],
                        kv_heads=cfg["kv_heads"], max_batch=max(batches), max_context=cfg["context"])
    st.bind_model(model)
    st.fill_kv(1)
    setup_s = time.perf_counter() - t0
    del model
    ts = torch.cuda.Stream()
    out = {"workload": "configs[4] synthetic decoder stack: 46 layers (3 dense NVFP4 MLP H2048 I10240, 42 NVFP4 MoE "
                       "c1 shapes, 1 BF16-expert MoE), BF16 GQA 32q/4kv/128 + q/k norm + RoPE, vocab 151552, "
                       "2048-token context, greedy decode, 1 GPU",
           "weights": "random init of the configuration's shapes; one attention block, dense MLP and NVFP4 MoE layer "
                      "generated on the host and bound into every layer of its kind (separate device copies)",
           "setup_s": setup_s, "per_batch": {}}
    L = cfg["context"]
    if cfg["layers"] != wl.STACK_CONFIGS["c4"]["layers"]:
        out["workload"] += f" [shortened to {cfg['layers']} layers]"
    for B in batches:
        rng = np.random.default_rng(B)
        tok = torch.from_numpy(rng.integers(0, cfg["vocab"], B).astype(np.int32)).cuda()
        pos = torch.full((B,), L - 1, dtype=torch.int32, device="cuda")
        nxt = torch.empty(B, dtype=torch.int32, device="cuda")
        for _ in range(2):
            st.decode(tok, pos, B, nxt, stream=ts.cuda_stream)
        st.sync(ts.cuda_stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=ts):
            st.decode(tok, pos, B, nxt, stream=ts.cuda_stream)
        for _ in range(max(1, args.warmup - 2)):
            graph.replay()
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 10))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(ts)
        with torch.cuda.stream(ts):
            for _ in range(steps):
                graph.replay()
        ev1.record(ts)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / steps
        st.sync(ts.cuda_stream)
        out["per_batch"][str(B)] = {"ms_per_step": ms, "tokens_per_s": B / (ms * 1e-3)}
        del graph
    st.close()
    return out


def run_decode_only(args, m, torch) -> dict:
    """The decode batch alone: warm-up, `steps` timed forwards, stage times."""
    lay, x_bits = wl.config_layer("c1")
    T, H, K = x_bits.shape[0], lay.hidden, lay.top_k
    layer = m.MoeLayer(H, lay.experts, K, lay.inter, lay.shared_inter, routed_scaling=lay.scaling,
                       swiglu_limit=lay.swiglu_limit, max_tokens=T)
    layer.bind_layer(lay)
    x = torch.from_numpy(x_bits.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        layer.forward(x, y, T, stream=stream)
    torch.cuda.synchronize()
    layer.profile(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        layer.forward(x, y, T, stream=stream)
    ev1.record()
    torch.cuda.synchronize()
    stages, nfw = layer.stage_times()
    layer.profile(False)
    layer.sync(stream)
    layer.close()
    ms = ev0.elapsed_time(ev1) / args.steps
    return {"workload": "c1 decode", "ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3),
            "stages_us": {k: 1e3 * v / max(nfw, 1) for k, v in stages.items()}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", action="store_true", help="skip the secondary prefill measurement")
    ap.add_argument("--no-stack", action="store_true", help="skip the configs[4] decoder-stack measurement")
    ap.add_argument("--expert-gemm", choices=["one_sm", "wide", "pair"], default="one_sm",
                    help="prefill: the expert GEMM form (nf_moe_set_expert_gemm); the default is the fastest measured")
    ap.add_argument("--stack-layers", type=int, default=None,
                    help="--only stack: a shorter stack of configs[4]'s shapes (profiling)")
    ap.add_argument("--stack-batches", type=int, nargs="*", default=None, help="--only stack: batch sizes to run")
    ap.add_argument("--only", choices=["decode", "prefill", "dense", "stack"],
                    help="time one workload alone (no e2e, CPU baseline or clock sampling); for profilers")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_env()
    if args.only:
        import torch

        m = load_module("nf_moe", PKG / "nf_moe.py")
        torch.cuda.set_device(local)
        if args.only == "decode":
            out = run_decode_only(args, m, torch)
        elif args.only == "dense":
            hbm_peak, bf16_peak, peak_src = peaks()
            out = run_dense(args, m, torch, hbm_peak, 4 * bf16_peak, peak_src)
        elif args.only == "stack":
            out = run_stack(args, m, torch, peaks()[0])
        else:
            _, bf16_peak, peak_src = peaks()
            out = run_prefill(args, m, torch, 4 * bf16_peak, bf16_peak, peak_src)
        print(json.dumps(out), flush=True)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
