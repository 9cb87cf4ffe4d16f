"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 and the built library; everything else runs
on the CPU (oracle checks against the reference's known answers, host
logic, and that the C-ABI library loads and exports its symbols).
"""
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
for sub in ("", "tests"):
    p = str(REPO / sub) if sub else str(REPO)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU and the built CUDA library")
