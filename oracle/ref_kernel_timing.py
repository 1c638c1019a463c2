"""TEST INFRASTRUCTURE: time the reference's own kernels (rebuilt for sm_100a
by oracle/Makefile) next to warp_decode_b200 on the same GPU and inputs.

Same method for both: every call replayed from a CUDA graph; "cold" = L2
flushed (256 MiB write + 256 MiB read) before each timed call, CUDA events
around the call only; "hot" = back-to-back replays of the same call (the
reference's published method, benchmark/bench.py:105-126).  Prints one JSON
object.

    python oracle/ref_kernel_timing.py [--batches 1,2,4,8,16,32,64] [--reps 50]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from warp_decode_b200 import warp_decode as wd  # noqa: E402
from warp_decode_b200 import workloads as W  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batches", default="1,2,4,8,16,32,64")
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--hot", type=int, default=200)
    args = ap.parse_args()
    L = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libwdref.so"))
    P, I_ = ctypes.c_void_p, ctypes.c_int
    L.wdref_gate_up.argtypes = [P, P, P, P, I_, I_, I_, I_, I_, P]
    L.wdref_down.argtypes = [P, P, P, P, P, I_, I_, I_, I_, I_, P]

    H, I, E, K = 4096, 192, 128, 8
    w_gu, w_dn = W.make_device_weights(H, I, E, 1234)
    fa = torch.empty(64 << 20, device="cuda")
    fb = torch.ones(64 << 20, device="cuda")
    fo = torch.empty((), device="cuda")

    def flush():
        fa.fill_(1.0)
        torch.sum(fb, dim=0, out=fo)

    stream = torch.cuda.Stream()

    def graph(fn):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        return g

    def cold(g):
        evs = []
        for _ in range(args.reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return float(np.mean([a.elapsed_time(b) for a, b in evs]) * 1e3)

    def hot(g):
        g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.hot):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / args.hot

    rows = []
    for B in [int(b) for b in args.batches.split(",")]:
        x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 1234 + B)
        h_r = torch.empty(B * K, I, dtype=torch.bfloat16, device="cuda")
        y_r = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")

        def ref_gu():
            L.wdref_gate_up(x.data_ptr(), w_gu.data_ptr(), ids.data_ptr(), h_r.data_ptr(), B, E, K, H,
                            I, torch.cuda.current_stream().cuda_stream)

        def ref_dn():
            L.wdref_down(h_r.data_ptr(), w_dn.data_ptr(), ids.data_ptr(), scale.data_ptr(),
                         y_r.data_ptr(), B, E, K, H, I, torch.cuda.current_stream().cuda_stream)

        def ref_e2e():
            ref_gu()
            ref_dn()

        def our_gu():
            return wd.moe_gate_up_3d_batched(x, w_gu, ids)

        def our_dn():
            return wd.moe_down_3d_batched(h_r, w_dn, ids, scale, B)

        def our_e2e():
            return wd.moe_ffn_3d_batched(x, w_gu, w_dn, ids, scale)

        U = W.unique_experts(ids.cpu().numpy())
        row = {"B": B, "unique_experts": U, "bytes": W.algorithmic_bytes(U, B, H, I, K)}
        for name, fn in [("ref_gate_up", ref_gu), ("ref_down", ref_dn), ("ref_e2e", ref_e2e),
                         ("ours_gate_up", our_gu), ("ours_down", our_dn), ("ours_e2e", our_e2e)]:
            g = graph(fn)
            row[name + "_cold_us"] = round(cold(g), 2)
            row[name + "_hot_us"] = round(hot(g), 2)
            del g
        rows.append(row)
        print(json.dumps(row), flush=True)
    print(json.dumps({"device": torch.cuda.get_device_name(), "rows": rows}))


if __name__ == "__main__":
    main()
