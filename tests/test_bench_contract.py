"""The benchmark's reference arm keeps its contract on the CPU: one JSON line
with the metric, unit, config and the cpu_baseline / e2e objects the driver
reads, timing the reference's own CPU path (oracle/_ref) on this host."""
import json
import subprocess
import sys

import pytest

from helpers import REPO, oracle


def test_reference_arm_prints_one_contract_line():
    if oracle().ref() is None:
        pytest.skip("reference sources not built (oracle/_ref)")
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["steps"] == 1 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "c1 decode" in d["config"]["workload"]


def test_cpu_legs_use_every_host_thread_under_torchrun():
    """torchrun exports OMP_NUM_THREADS=1 to every rank; bench.py overrides it
    with the process's host threads before the oracle loads, so the reference
    arm is timed on all cores at every N."""
    import os

    env = dict(os.environ, OMP_NUM_THREADS="1", RANK="0", WORLD_SIZE="2", LOCAL_RANK="0")
    code = ("import os, sys; sys.path.insert(0, %r); import bench; "
            "print(os.environ['OMP_NUM_THREADS'], bench.cpu_threads())") % str(REPO)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    omp, n = r.stdout.split()
    assert int(omp) == int(n) == len(os.sched_getaffinity(0))


def test_ep_roofline_counts_per_rank_bytes():
    """At N > 1 a rank streams only its own experts that received rows: the
    per-rank bytes sum to the whole layer's expert weights once, and rank 0's
    gate/up bytes never exceed the single-GPU figure for the same routes."""
    import numpy as np

    sys.path.insert(0, str(REPO))
    import bench

    lay, _ = bench.wl.config_layer("c1")
    rng = np.random.default_rng(5)
    E, K = lay.experts, lay.top_k
    for world in (2, 4, 8):
        idx_all = [np.stack([rng.choice(E, K, replace=False) for _ in range(64)]) for _ in range(world)]
        per = [bench.ep_rank_bytes(lay, idx_all, r, world) for r in range(world)]
        active = np.unique(np.concatenate([a.ravel() for a in idx_all])).size
        assert sum(p["active_owned"] for p in per) == active
        assert sum(p["rows_received"] for p in per) == world * 64 * K
        one = bench.decode_bytes(lay, active, world * 64)
        assert per[0]["gate_up"] < one["gate_up"]
        H, I = lay.hidden, lay.inter
        w_all = active * (3 * I * H // 2 + 3 * I * H // 16)
        shared_router = 3 * lay.shared_inter * H * 2 + E * H * 2 + E * 4
        io = 64 * H * 6
        exch = world * 64 * K * H * 8
        assert sum(p["layer"] for p in per) == w_all + world * (shared_router + io) + exch


def test_replica_choice_lowers_the_busiest_rank():
    """choose_replicas picks hot experts only while replicating them lowers the
    busiest rank's pick load: a skewed count matrix (expert 0 hot, owned by
    rank 0) gets expert 0 replicated and a balanced one gets nothing."""
    import numpy as np

    sys.path.insert(0, str(REPO))
    import bench

    world, E = 2, 8
    counts = np.full((world, E), 10, dtype=np.int64)
    counts[:, 0] = 500  # every rank's tokens pick expert 0 (rank 0 owns 0-3)
    reps = bench.choose_replicas(counts, E // world)
    assert 0 in reps

    def busiest(rs):
        tot = counts.sum(0)
        load = np.zeros(world)
        for e in range(E):
            if e in rs:
                load += counts[:, e]
            else:
                load[e // (E // world)] += tot[e]
        return load.max()

    assert busiest(set(reps)) < busiest(set())
    assert bench.choose_replicas(np.full((world, E), 10, dtype=np.int64), E // world) == []
