"""Shared helpers for the tests: module loading by path (the package folder's
name is not a Python identifier), GPU availability, tolerance checks."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "ninfer_nvfp4_glm-5.3_flash_2x_dgxspark_b200"

# Layer-output tolerance of the benchmark's correctness bar.
MAX_ABS = 2e-2
MIN_COS = 0.9995


def load_module(name: str, path: Path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def nfm():
    return load_module("nf_moe", PKG / "nf_moe.py")


def workload():
    return load_module("nf_workload", PKG / "workload.py")


def oracle():
    return load_module("nf_oracle_py", REPO / "oracle" / "oracle.py")


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def assert_close(got: np.ndarray, want: np.ndarray, max_abs: float = MAX_ABS, min_cos: float = MIN_COS, what: str = ""):
    err = float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) if got.size else 0.0
    cos = cosine(got, want) if got.size else 1.0
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert err <= max_abs, f"{what}: max-abs {err:.3e} > {max_abs:.1e}"
    assert cos >= min_cos, f"{what}: cosine {cos:.6f} < {min_cos}"
    return err, cos
