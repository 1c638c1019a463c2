"""Shared pytest setup: the `gpu` marker and fixture helpers.

Tests marked ``gpu`` need a CUDA device and the built native library; the
rest run on any CPU machine.  The driver runs ``-m "not gpu"`` on CPU and
``-m gpu`` on a B200.
"""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_cases():
    return json.loads((GOLDEN / "golden.json").read_text())["cases"]


_golden_arrays = None


def golden_array(key: str) -> np.ndarray:
    global _golden_arrays
    if _golden_arrays is None:
        _golden_arrays = dict(np.load(GOLDEN / "golden.npz"))
    return _golden_arrays[key]


def golden_inputs(case: dict, full: bool = False) -> dict:
    from warp_decode_b200.workloads import input_digest, make_host_inputs

    inp = make_host_inputs(case["B"], case["hidden"], case["inter"], case["E"], case["topk"],
                           seed=case["seed"], routing=case["routing"], x_std=case["x_std"],
                           w_std=case["w_std"], wd_std=case["wd_std"], full=full)
    assert input_digest(inp) == case["sha256"], "input generator drifted from the fixtures"
    return inp


def bf16_close(a_u16, b_u16, rtol, atol):
    """Elementwise |a-b| <= atol + rtol*|b| on bf16 bit arrays; returns (ok, max_abs_diff)."""
    from oracle.moe_ref import bf16_to_f32

    a = bf16_to_f32(a_u16).astype(np.float64)
    b = bf16_to_f32(b_u16).astype(np.float64)
    d = np.abs(a - b)
    return bool(np.all(d <= atol + rtol * np.abs(b))), float(d.max(initial=0.0))
