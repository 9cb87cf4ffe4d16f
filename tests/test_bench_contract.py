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
