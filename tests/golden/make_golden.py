"""Generate the golden fixtures that pin the oracle to the reference itself.

Runs in a container where the reference repository (Religious-J/warp_decode)
is mounted read-only; it is never needed at test time.  For every case it

1. builds the inputs with ``warp_decode_b200.workloads.make_host_inputs``
   (numpy PCG64, so any machine regenerates them bit for bit; weights exist
   only for the experts the routing touches, the rest are zero; a SHA-256 of
   the inputs is stored to detect drift),
2. runs the reference's own PyTorch functions on CPU tensors:
   ``reference_gate_up`` (tests/test_gate_up_correctness.py:19-43) and
   ``reference_down`` (tests/test_down_correctness.py:14-35), imported from the
   reference test modules with a stub standing in for the compiled
   ``warp_decode`` extension (the tests import it at module level), and
3. runs the reference's FP32 formula, the statements of
   tests/test_benchmark_reference.py:36-43, taken from that file's syntax
   tree and executed unmodified (the rest of that file needs SGLang).

Outputs are stored as bf16 bit patterns in ``golden.npz`` with a JSON index.

Usage:  python tests/golden/make_golden.py [--ref /path/to/reference]
"""
from __future__ import annotations

import argparse
import os
import ast
import importlib.util
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from warp_decode_b200.workloads import input_digest, make_host_inputs  # noqa: E402

# (name, B, E, topk, hidden, inter, routing, x_std, w_std, wd_std, seed)
# The first twelve follow the reference's own test cases
# (tests/test_gate_up_correctness.py:79-87, tests/test_down_correctness.py:68-76:
#  x = randn*0.1, w = randn*0.05, randint routing); the rest use the benchmark
# configurations' distributions (x ~ N(0,1), W ~ N(0, fan_in^-1/2)).
CASES = [
    ("gu_ref_1", 1, 4, 2, 256, 8, "randint", 0.1, 0.05, 0.05, 101),
    ("gu_ref_2", 2, 8, 2, 512, 16, "randint", 0.1, 0.05, 0.05, 102),
    ("gu_ref_3", 4, 16, 4, 1024, 64, "randint", 0.1, 0.05, 0.05, 103),
    ("gu_ref_4", 8, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 104),
    ("gu_ref_5", 16, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 105),
    ("gu_ref_6", 64, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 106),
    ("dn_ref_1", 1, 4, 2, 256, 64, "randint", 0.1, 0.05, 0.05, 201),
    ("dn_ref_2", 2, 8, 4, 512, 64, "randint", 0.1, 0.05, 0.05, 202),
    ("dn_ref_3", 4, 16, 4, 1024, 128, "randint", 0.1, 0.05, 0.05, 203),
    ("dn_ref_4", 8, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 204),
    ("dn_ref_5", 16, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 205),
    ("dn_ref_6", 64, 16, 8, 4096, 192, "randint", 0.1, 0.05, 0.05, 206),
    # FP32-reference cases (tests/test_benchmark_reference.py:73-75 shapes, E reduced
    # where the CPU reference would gather gigabytes)
    ("e2e_1", 1, 4, 1, 256, 64, "uniform", 1.0, None, None, 301),
    ("e2e_2", 3, 8, 2, 512, 128, "uniform", 1.0, None, None, 302),
    ("e2e_qwen_b1", 1, 128, 8, 4096, 192, "uniform", 1.0, None, None, 303),
    ("e2e_qwen_b8", 8, 32, 8, 4096, 192, "uniform", 1.0, None, None, 304),
    ("e2e_qwen_b32", 32, 32, 8, 4096, 192, "uniform", 1.0, None, None, 305),
    ("e2e_i384", 4, 32, 8, 4096, 384, "uniform", 1.0, None, None, 306),
    ("e2e_dsv3_zipf", 8, 256, 8, 7168, 256, "zipf", 1.0, None, None, 307),
    ("e2e_q30b", 4, 32, 8, 2048, 768, "uniform", 1.0, None, None, 308),
]


def _load_reference_tests(ref: Path):
    """Import reference_gate_up / reference_down without building CUDA code."""
    stub = types.ModuleType("warp_decode")
    stub.warp_decode = None  # the compiled extension; not used by the references
    sys.modules["warp_decode"] = stub
    mods = {}
    for name in ("test_gate_up_correctness", "test_down_correctness"):
        spec = importlib.util.spec_from_file_location(f"_ref_{name}", ref / "tests" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["test_gate_up_correctness"].reference_gate_up, mods["test_down_correctness"].reference_down


def _load_fp32_formula(ref: Path):
    """Compile the FP32 reference statements of test_benchmark_reference.run_case."""
    path = ref / "tests" / "test_benchmark_reference.py"
    tree = ast.parse(path.read_text())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "run_case")
    body = []
    started = False
    for stmt in fn.body:
        src = ast.unparse(stmt)
        if src.startswith("selected_gu ="):
            started = True
        if started:
            body.append(stmt)
            if src.startswith("ref ="):
                break
    if not body or not ast.unparse(body[-1]).startswith("ref ="):
        raise RuntimeError("FP32 reference statements not found")
    mod = ast.Module(body=body, type_ignores=[])
    code = compile(mod, str(path), "exec")
    lines = (body[0].lineno, body[-1].end_lineno)

    def run(gu, dn, x, ids, scale, B, topk, hidden):
        ns = {"torch": torch, "gu": gu, "dn": dn, "x": x, "ids": ids, "scale": scale,
              "B": B, "topk": topk, "hidden": hidden}
        exec(code, ns)
        return ns["ref_buffer"], ns["ref"]

    return run, lines


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("WARP_DECODE_REFERENCE"),
                    help="checkout of Religious-J/warp_decode (default: $WARP_DECODE_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref or WARP_DECODE_REFERENCE must name the reference checkout")
    ref = Path(args.ref)
    torch.set_num_threads(8)
    ref_gate_up, ref_down = _load_reference_tests(ref)
    fp32_ref, fp32_lines = _load_fp32_formula(ref)

    arrays = {}
    index = {"generator": "warp_decode_b200.workloads.make_host_inputs",
             "fp32_formula": f"tests/test_benchmark_reference.py:{fp32_lines[0]}-{fp32_lines[1]}",
             "torch": torch.__version__, "cases": []}
    for (name, B, E, K, H, I, routing, xs, ws, wds, seed) in CASES:
        inp = make_host_inputs(B, H, I, E, K, seed=seed, routing=routing, x_std=xs,
                               w_std=ws, wd_std=wds, full=True)
        x = torch.from_numpy(inp["x"].view(np.int16)).view(torch.bfloat16)
        gu = torch.from_numpy(inp["w_gate_up"].view(np.int16)).view(torch.bfloat16)
        dn = torch.from_numpy(inp["w_down"].view(np.int16)).view(torch.bfloat16)
        ids = torch.from_numpy(inp["topk_ids"])
        scale = torch.from_numpy(inp["topk_scale"])
        # reference_gate_up / reference_down: bf16 bmm semantics
        h_bf16 = ref_gate_up(x, gu, ids)
        y_bf16 = ref_down(h_bf16, dn, ids, scale)
        # FP32 formula: h with the bf16 boundary, y from the FP32 h path
        h_fp32, y_fp32 = fp32_ref(gu, dn, x, ids, scale, B, K, H)
        arrays[f"{name}/h_bf16"] = _bits(h_bf16)
        arrays[f"{name}/y_bf16"] = _bits(y_bf16)
        arrays[f"{name}/h_fp32"] = _bits(h_fp32)
        arrays[f"{name}/y_fp32"] = _bits(y_fp32)
        index["cases"].append(dict(name=name, B=B, E=E, topk=K, hidden=H, inter=I,
                                   routing=routing, x_std=xs, w_std=ws, wd_std=wds, seed=seed,
                                   sha256=input_digest(inp)))
        print(f"{name}: B={B} E={E} K={K} H={H} I={I} {routing}", flush=True)
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(index, indent=1) + "\n")
    print("wrote", HERE / "golden.npz")


if __name__ == "__main__":
    main()
