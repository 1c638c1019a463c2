#!/usr/bin/env python
"""MoE FFN decode benchmark: us/call at B = 1..64 and achieved HBM bandwidth.

Metric and workload: MoE FFN us/call at B=1-64 and achieved
HBM TB/s vs B200 peak, on the Qwen3-235B-A22B MoE FFN TP=8 shard
(hidden 4096, inter 192 per GPU, 128 experts, top-8, bf16, uniform distinct
routing, softmax top-k weights, weights ~ N(0, fan_in^-1/2), x ~ N(0,1)).

One *step* = one end-to-end MoE FFN call (gate_up -> down, the reference
bench's e2e, benchmark/bench.py:251-256 of Religious-J/warp_decode) at every
batch size of the sweep B in {1,2,4,8,16,32,64}.  Every call is replayed from
a CUDA graph (the reference's timing method, bench.py:105-126) with L2
flushed before it (a 256 MiB write followed by a 256 MiB read, outside the
timed window), timed with CUDA events on the launching stream.  value = mean
us per call over the sweep, max over ranks.

--gpus N > 1 (torchrun, one process per GPU): each rank holds a 192-wide
slice of an inter = 192*N FFN (at N = 8 the full-width Qwen3-235B FFN split
TP=8); the call ends with one NCCL all-reduce of the FP32 partial [B, 4096]
output, then the bf16 cast.  Per-GPU work is fixed: "scaling": "weak".

--workload selects another BASELINE configuration at the same method:
qwen3_235b_full (inter 1536 split over the N GPUs: strong scaling), dsv3_tp8
(hidden 7168, 256 experts, Zipf routing), qwen3_30b_mxfp8 (MXFP8 weights,
one GPU).  The default is the headline workload above.

--impl reference times the reference's PyTorch path (gather + bf16 bmm,
tests/test_gate_up_correctness.py:19-43 / tests/test_down_correctness.py:14-35)
on the host cores, via the CPU port in oracle/torch_port.py.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

SWEEP = (1, 2, 4, 8, 16, 32, 64)
WORKLOAD = "qwen3_235b_tp8"
METRIC = "MoE FFN µs/call at B=1–64 and achieved HBM TB/s vs B200 peak, 1/2/4/8 GPU"
UNIT = "us/call"
L2_FLUSH_BYTES = 256 << 20
FALLBACK_HBM_GBS = 6650.0
# Published reference numbers (NVIDIA H20, L2-warm graph replay; README.md:80-90)
PUBLISHED_H20_E2E_US = {1: 23.2, 2: 35.0, 4: 51.1, 8: 87.8, 16: 143.0, 32: 268.2, 64: 518.7}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default=WORKLOAD,
                   choices=["qwen3_235b_tp8", "qwen3_235b_full", "dsv3_tp8", "qwen3_30b_mxfp8"],
                   help="BASELINE configuration (default: the headline TP=8 shard)")
    p.add_argument("--batches", default=None, help="comma-separated B values (default: the workload's)")
    p.add_argument("--hot-iters", type=int, default=200, help="graph replays for the L2-warm numbers")
    p.add_argument("--kernel-reps", type=int, default=30, help="cold reps per kernel measurement")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true", help="headline only (no per-kernel/e2e legs)")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--allreduce", choices=["fused", "nccl"], default="fused",
                   help="N > 1: all-reduce fused into the down kernel, or NCCL after it")
    p.add_argument("--profile-once", action="store_true",
                   help="one eager e2e call per batch size, no timing (for ncu captures)")
    p.add_argument("--no-others", action="store_true",
                   help="skip the BASELINE configs[3] / configs[4] legs (DeepSeek-V3 Zipf, MXFP8)")
    p.add_argument("--no-tp-full", action="store_true",
                   help="skip the BASELINE configs[2] leg (full-width inter 1536 split over the N GPUs)")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def measured_peaks():
    """HBM copy bandwidth measured on this pool (MEASURED_PEAKS.json next to this file)."""
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# clocks (NVML, the library nvidia-smi reads)
# ---------------------------------------------------------------------------
_REASONS = [(0x1, "gpu_idle"), (0x2, "applications_clocks_setting"), (0x4, "sw_power_cap"),
            (0x8, "hw_slowdown"), (0x10, "sync_boost"), (0x20, "sw_thermal_slowdown"),
            (0x40, "hw_thermal_slowdown"), (0x80, "hw_power_brake_slowdown"),
            (0x100, "display_clock_setting")]


class ClockSampler:
    """Samples SM clock and clock-event reasons of this process's GPU every 5 ms."""

    def __init__(self, device_index: int):
        self.samples = []
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml as N

            N.nvmlInit()
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            try:
                h = N.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                h = N.nvmlDeviceGetHandleByIndex(device_index)
            self._N, self._h = N, h
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - depends on the box
            self.error = f"nvml unavailable: {e}"

    def _reasons(self):
        N, h = self._N, self._h
        fn = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(N, "nvmlDeviceGetCurrentClocksThrottleReasons")
        return fn(h)

    def _run(self):
        N, h = self._N, self._h
        while not self._stop.is_set():
            try:
                self.samples.append((time.perf_counter(), N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM),
                                     self._reasons()))
            except Exception as e:  # pragma: no cover
                self.error = str(e)
                return
            self._stop.wait(0.005)

    def start(self):
        if self.error is None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self, t0: float, t1: float) -> dict:
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:
            win = self.samples
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.error or "no samples"}
        mask = 0
        for s in win:
            mask |= s[2]
        reasons = [n for b, n in _REASONS if mask & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[1] for s in win), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class L2Flush:
    """Evict L2: write then read a buffer twice the size of L2 (126 MB on B200)."""

    def __init__(self, device):
        import torch

        n = L2_FLUSH_BYTES // 4
        self.a = torch.empty(n, dtype=torch.float32, device=device)
        self.b = torch.ones(n, dtype=torch.float32, device=device)
        self.out = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self):
        import torch

        self.a.fill_(1.0)
        torch.sum(self.b, dim=0, out=self.out)


def fp32_reference_partial(x, w_gu, w_dn, ids, scale):
    """This rank's FP32 partial [B, H] of the FFN by the FP32 formula of the
    reference (tests/test_benchmark_reference.py:36-43): projections in
    float64 rounded to FP32, silu(g)*u in FP32, h rounded to bf16 (the bf16
    boundary at h), down projections in float64 rounded to FP32, times the
    top-k weight, summed over the slots in FP32.  Plain torch on the device
    (a checker, not the product): the sum over ranks of these partials is the
    unsharded FFN, because silu(g)*u is elementwise in `inter`."""
    import torch

    B, K = ids.shape
    I = w_gu.shape[1] // 2
    flat = ids.reshape(-1).long()
    xs = x.double().repeat_interleave(K, dim=0)                      # [B*K, H]
    proj = torch.bmm(w_gu[flat].double(), xs.unsqueeze(-1)).squeeze(-1).float()
    g, u = proj[:, :I], proj[:, I:]
    h = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)          # [B*K, I]
    p = torch.bmm(w_dn[flat].double(), h.double().unsqueeze(-1)).squeeze(-1).float()
    p = p.view(B, K, -1) * scale.unsqueeze(-1)
    y = torch.zeros_like(p[:, 0])
    for s_ in range(K):
        y = y + p[:, s_]
    return y


def check_parity(cases, e2e_call, nccl_call, w_gu, w_dn, world, fused, tol=1e-2):
    """Outputs of the timed path against the FP32 reference (summed over the
    ranks with NCCL when world > 1) at rtol = atol = tol; at world > 1 also
    against the NCCL all-reduce path, the same bits on every rank, and the
    same bits from both fused exchange shapes.  Returns the JSON record."""
    import torch
    import torch.distributed as dist

    recs, ok_all = [], True
    for c in cases:
        y = e2e_call(c)
        ref = fp32_reference_partial(c.x, w_gu, w_dn, c.ids, c.scale)
        if world > 1:
            dist.all_reduce(ref)
        ref_bf = ref.to(torch.bfloat16).float()
        yf = y.float()
        d_ref = (yf - ref_bf).abs()
        ok = bool((d_ref <= tol + tol * ref_bf.abs()).all().item())
        rec = {"B": c.B, "max_abs_diff_vs_fp32_ref": float(d_ref.max().item())}
        if world > 1:
            yn = nccl_call(c).float()
            d_n = (yf - yn).abs()
            ok &= bool((d_n <= tol + tol * yn.abs()).all().item())
            rec["max_abs_diff_vs_nccl"] = float(d_n.max().item())
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            same = all(torch.equal(gathered[0].view(torch.int16), g.view(torch.int16))
                       for g in gathered)
            rec["identical_on_all_ranks"] = same
            ok &= same
            if fused is not None and fused.applies(c.B):
                shapes_same = True
                for mode in (1, 2):
                    fused.set_exchange(mode)
                    shapes_same &= torch.equal(e2e_call(c).view(torch.int16), y.view(torch.int16))
                fused.set_exchange(0)
                rec["exchange_shapes_identical"] = shapes_same
                ok &= shapes_same
        torch.cuda.synchronize()
        flag = torch.tensor([1 if ok else 0], device=y.device)
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        rec["ok"] = bool(flag.item())
        ok_all &= rec["ok"]
        recs.append(rec)
    return {"tol": {"rtol": tol, "atol": tol}, "reference": "FP32 formula of "
            "tests/test_benchmark_reference.py:36-43 on the device (torch, float64 projections)"
            + (", partials summed over the ranks" if world > 1 else ""),
            "cases": recs, "ok": ok_all}


def run_ours(args, rank, local_rank, world):
    import numpy as np
    import torch
    import torch.distributed as dist

    from warp_decode_b200 import warp_decode as wd
    from warp_decode_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    cfg = W.CONFIGS[args.workload]
    batches = [int(b) for b in args.batches.split(",")] if args.batches else list(cfg.batches)
    mx = cfg.weights == "mxfp8"
    if mx and world > 1:
        raise SystemExit("bench.py: the MXFP8 workload runs on one GPU")
    # qwen3_235b_full: the fixed full-width FFN split over the ranks (strong
    # scaling); the shard workloads: every rank one shard-sized slice (weak).
    strong = args.workload == "qwen3_235b_full"
    H, E, K = cfg.hidden, cfg.E, cfg.topk
    I = cfg.inter_full // world if strong else cfg.inter

    w_gu, w_dn = W.make_device_weights(H, I, E, args.seed + 7919 * rank, device=dev)
    if mx:
        from warp_decode_b200.mxfp8 import quantize_mxfp8

        gq, gs = quantize_mxfp8(w_gu)
        dq, ds = quantize_mxfp8(w_dn)
        del w_gu, w_dn
        torch.cuda.empty_cache()

        def gate_up(x, ids):
            return wd.moe_gate_up_3d_batched_mxfp8(x, gq, gs, ids)

        def down(h, ids, sc, B):
            return wd.moe_down_3d_batched_mxfp8(h, dq, ds, ids, sc, B)

        def ffn(x, ids, sc):
            return down(gate_up(x, ids), ids, sc, x.shape[0])
    else:
        def gate_up(x, ids):
            return wd.moe_gate_up_3d_batched(x, w_gu, ids)

        def down(h, ids, sc, B):
            return wd.moe_down_3d_batched(h, w_dn, ids, sc, B)

        def ffn(x, ids, sc):
            # one call: single cooperative launch where it applies, else the two kernels
            return wd.moe_ffn_3d_batched(x, w_gu, w_dn, ids, sc)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(device=dev)

    class Case:
        pass

    cases = {}
    for B in batches:
        c = Case()
        c.B = B
        c.x, c.ids, c.scale = W.make_device_activations(B, H, E, K, cfg.routing, args.seed + B, device=dev)
        c.U = W.unique_experts(c.ids.cpu().numpy())
        c.bytes = W.algorithmic_bytes(c.U, B, H, I, K, cfg.weights)
        cases[B] = c

    fused = None
    if world > 1 and args.allreduce == "fused":
        from warp_decode_b200.tp import FusedAllReduce

        fused = FusedAllReduce(H, max_tokens=64)

    def nccl_call(c):
        h = wd.moe_gate_up_3d_batched(c.x, w_gu, c.ids)
        part = wd.moe_down_3d_batched_partial(h, w_dn, c.ids, c.scale, c.B)
        dist.all_reduce(part)
        return part.to(torch.bfloat16)

    def e2e_call(c):
        if world == 1:
            return ffn(c.x, c.ids, c.scale)
        if fused is not None and fused.applies(c.B):
            # one launch (FFN + exchange) for B*topk <= 32, else gate_up + down
            return fused.ffn(c.x, w_gu, w_dn, c.ids, c.scale)
        return nccl_call(c)

    if args.profile_once:
        # One eager call per batch size and nothing else (profiler captures:
        # the k-th launch of a kernel is the k-th batch size's call).
        for B in batches:
            e2e_call(cases[B])
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
            if fused is not None:
                fused.close()
            dist.destroy_process_group()
        return 0

    # Correctness of the timed path before timing it (every rank, same order).
    parity = None
    if not mx:
        pcases = [cases[B] for B in (1, 8, 64) if B in cases] or [cases[batches[0]]]
        parity = check_parity(pcases, e2e_call, nccl_call, w_gu, w_dn, world, fused)
        torch.cuda.empty_cache()

    def capture(fn):
        """CUDA graph of one call, and how many of the library's kernels it holds."""
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = wd.launch_count()
        with torch.cuda.graph(g, stream=stream):
            out = fn()
        return g, out, wd.launch_count() - n0

    launches = {}
    for c in cases.values():
        c.g_e2e, c.y, launches[c.B] = capture(lambda c=c: e2e_call(c))
        c.g_gu, c.h, _ = capture(lambda c=c: gate_up(c.x, c.ids))
        c.g_dn, _, _ = capture(lambda c=c: down(c.h, c.ids, c.scale, c.B))
        c.g_split = c.g_nccl = None
        if world > 1 and not args.no_extras:
            # the unfused path of the same call (partial down, NCCL all-reduce,
            # bf16 cast) for the per-B fused-vs-NCCL comparison
            c.g_nccl, _, _ = capture(lambda c=c: nccl_call(c))
        if world == 1 and not mx:
            c.g_split, _, _ = capture(lambda c=c: down(gate_up(c.x, c.ids), c.ids, c.scale, c.B))
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # ---- headline: K steps, each = one cold e2e call per batch size ----
    nB = len(batches)
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in batches] for _ in range(args.steps)]
    cur = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        for B in batches:
            flush()
            cases[B].g_e2e.replay()
    sampler = ClockSampler(local_rank).start()
    barrier()
    torch.cuda.synchronize()
    t_start = time.perf_counter()
    for s in range(args.steps):
        for i, B in enumerate(batches):
            flush()
            evs[s][i][0].record(cur)
            cases[B].g_e2e.replay()
            evs[s][i][1].record(cur)
    torch.cuda.synchronize()
    barrier()
    t_end = time.perf_counter()
    sampler.stop()
    per_call = np.array([[evs[s][i][0].elapsed_time(evs[s][i][1]) for i in range(nB)]
                         for s in range(args.steps)])  # ms
    total_ms = torch.tensor([per_call.sum()], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    ms_per_step = total_ms / args.steps
    value_us = total_ms * 1000.0 / (args.steps * nB)
    per_b_us = {B: float(per_call[:, i].mean() * 1000.0) for i, B in enumerate(batches)}
    clocks = sampler.summary(t_start, t_end)

    peak_gbs, peak_kind = measured_peaks()
    sweep = []
    roofline = None
    e2e = None
    if not args.no_extras:
        def cold_time(graph, reps):
            ts = []
            for _ in range(reps):
                flush()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(cur)
                graph.replay()
                b.record(cur)
                ts.append((a, b))
            torch.cuda.synchronize()
            return float(np.mean([a.elapsed_time(b) for a, b in ts]) * 1000.0)

        def hot_time(graph, iters):
            graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            for _ in range(iters):
                graph.replay()
            b.record(cur)
            torch.cuda.synchronize()
            return a.elapsed_time(b) * 1000.0 / iters

        gu_bytes = gu_time = 0.0
        for B in batches:
            c = cases[B]
            t_gu = cold_time(c.g_gu, args.kernel_reps)
            t_dn = cold_time(c.g_dn, args.kernel_reps)
            t_hot = hot_time(c.g_e2e, args.hot_iters)
            t_split = cold_time(c.g_split, args.kernel_reps) if c.g_split is not None else None
            t_nccl = cold_time(c.g_nccl, args.kernel_reps) if c.g_nccl is not None else None
            gu_bytes += c.bytes["gate_up"]
            gu_time += t_gu
            sweep.append({
                "B": B, "unique_experts": c.U, "e2e_us": round(per_b_us[B], 2),
                "e2e_launches": launches[B],
                "e2e_hot_us": round(t_hot, 2), "gate_up_us": round(t_gu, 2), "down_us": round(t_dn, 2),
                "two_call_e2e_us": round(t_split, 2) if t_split is not None else None,
                "nccl_e2e_us": round(t_nccl, 2) if t_nccl is not None else None,
                "exchange": exchange_record(fused, B, H, world),
                "bytes_e2e": c.bytes["e2e"],
                "e2e_tbs": round(c.bytes["e2e"] / (per_b_us[B] * 1e-6) / 1e12, 3),
                "e2e_frac": round(c.bytes["e2e"] / (per_b_us[B] * 1e-6) / 1e9 / peak_gbs, 3),
                "gate_up_frac": round(c.bytes["gate_up"] / (t_gu * 1e-6) / 1e9 / peak_gbs, 3),
                "down_frac": round(c.bytes["down"] / (t_dn * 1e-6) / 1e9 / peak_gbs, 3),
                "published_h20_hot_e2e_us": (PUBLISHED_H20_E2E_US.get(B)
                                             if args.workload == WORKLOAD else None),
            })
        # Roofline of the dominant kernel of the e2e path: the kernel choice
        # of each call (wd_moe_ffn_3d_batched_kernels), its share of the
        # sweep's time; a single-launch choice is one kernel, so its CUDA-event
        # time is that kernel's launch duration and its bytes the call's.
        from warp_decode_b200 import capi

        kinds = {}
        if world == 1 and not mx:
            for B in batches:
                kinds[B] = capi.ffn_kernels(B, E, K, H, I)
        share = {}
        for B, k in kinds.items():
            share[k] = share.get(k, 0.0) + per_b_us[B]
        dom = max(share, key=share.get) if share else None
        traffic = None
        if dom in (capi.FFN_KERNELS_TC_SINGLE, capi.FFN_KERNELS_SIMT_SINGLE):
            bs = [B for B in batches if kinds[B] == dom]
            kbytes = sum(cases[B].bytes["e2e"] for B in bs)
            ktime = sum(per_b_us[B] for B in bs)
            kname = ("moe_ffn_tc_kernel (tensor-core single launch)"
                     if dom == capi.FFN_KERNELS_TC_SINGLE else "moe_ffn_kernel (SIMT single launch)")
            fname = "ffn_tc_dram_traffic.json" if dom == capi.FFN_KERNELS_TC_SINGLE else None
            method = (f"sum of algorithmic e2e bytes over the calls this kernel serves (B = "
                      f"{', '.join(map(str, bs))}; one launch each) / sum of their cold CUDA-event "
                      f"durations; {100.0 * ktime / sum(per_b_us.values()):.0f} % of the sweep's time")
        else:
            bs = list(batches)
            kbytes, ktime = gu_bytes, gu_time
            kname = ("gate_up (moe_gate_up_kernel<e4m3>, MXFP8 weights)" if mx else
                     "gate_up (moe_gate_up_kernel B<16, moe_gate_up_tc_kernel B>=16)")
            fname = None
            method = ("sum of algorithmic gate_up bytes over the sweep / sum of cold per-launch "
                      "CUDA-event durations (one launch per batch size)")
        achieved = kbytes / (ktime * 1e-6) / 1e9
        if fname and (ROOT / "profiles" / fname).exists() and args.workload == WORKLOAD:
            try:
                t = json.loads((ROOT / "profiles" / fname).read_text())
                per = [t["per_batch"][str(B)] for B in bs if str(B) in t["per_batch"]]
                if len(per) == len(bs):
                    traffic = sum(per) / len(bs)
            except Exception:
                traffic = None
        roofline = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1),
                    "peak": peak_gbs, "peak_kind": peak_kind, "unit": "GB/s",
                    "frac": round(achieved / peak_gbs, 4),
                    "alg_bytes_per_launch": kbytes / len(bs), "traffic": traffic,
                    "method": method}

        # ---- end to end through the public API with host buffers ----
        # x, topk_ids and topk_scale of a call sit in one pinned host buffer
        # and go to the device in one copy (views of one device buffer).
        packed = {}
        for B in batches:
            c = cases[B]
            parts = [c.x.cpu().view(torch.uint8).reshape(-1), c.ids.cpu().view(torch.uint8).reshape(-1),
                     c.scale.cpu().view(torch.uint8).reshape(-1)]
            host = torch.cat(parts).pin_memory()
            dbuf = torch.empty_like(host, device=dev)
            xb, ib = parts[0].numel(), parts[1].numel()
            xd = dbuf[:xb].view(torch.bfloat16).view(B, H)
            idd = dbuf[xb:xb + ib].view(torch.int32).view(B, K)
            scd = dbuf[xb + ib:].view(torch.float32).view(B, K)
            xh = host[:xb].view(torch.bfloat16).view(B, H)
            idh = host[xb:xb + ib].view(torch.int32).view(B, K)
            sch = host[xb + ib:].view(torch.float32).view(B, K)
            packed[B] = (host, dbuf, xd, idd, scd, torch.empty(B, H, dtype=torch.bfloat16).pin_memory(),
                         (xh, idh, sch))
        h2d = sum(B * H * 2 + B * K * 8 for B in batches)
        d2h = sum(B * H * 2 for B in batches)
        reps = max(5, min(args.steps, 30))

        def api_call(B, xd, idd, scd):
            if world == 1:
                return ffn(xd, idd, scd)
            if fused is not None and fused.applies(B):
                return fused.ffn(xd, w_gu, w_dn, idd, scd)
            h = wd.moe_gate_up_3d_batched(xd, w_gu, idd)
            y = wd.moe_down_3d_batched_partial(h, w_dn, idd, scd, B)
            dist.all_reduce(y)
            return y.to(torch.bfloat16)

        def e2e_step(B):
            """One step through the public API with host buffers: inputs in
            and y out by the library's copy kernel (wd_copy_ranges), the FFN
            between (moe_ffn_3d_batched_host does all three at N = 1)."""
            host, dbuf, xd, idd, scd, yh, (xh, idh, sch) = packed[B]
            if world == 1 and not mx:
                return wd.moe_ffn_3d_batched_host(xh, w_gu, w_dn, idh, sch, out=yh)
            wd.copy_ranges([host], [dbuf])
            y = api_call(B, xd, idd, scd)
            wd.copy_ranges([y], [yh])
            return yh

        def timed(fn):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            fn()
            b.record(cur)
            return a, b

        # Per call, cold timings of the same step (L2 flushed first): the e2e
        # step itself and, at N = 1, its parts: the two transfers alone by the
        # copy kernel and by the copy engine (non_blocking torch copies: the
        # packed inputs in, a [B, H] bf16 buffer out), and the eager API call
        # alone on device-resident inputs.  Only the first enters `value`.
        e2e_ts = []
        parts_ts = {B: {"copies": [], "copies_dma": [], "eager_call": []} for B in batches}
        for r in range(reps + 2):
            row = []
            for B in batches:
                host, dbuf, xd, idd, scd, yh, _ = packed[B]
                row.append(timed(lambda: e2e_step(B)))
                if world == 1:
                    y = cases[B].y
                    ev = {"copies": timed(lambda: (wd.copy_ranges([host], [dbuf]),
                                                   wd.copy_ranges([y], [yh]))),
                          "copies_dma": timed(lambda: (dbuf.copy_(host, non_blocking=True),
                                                       yh.copy_(y, non_blocking=True))),
                          "eager_call": timed(lambda: api_call(B, xd, idd, scd))}
                    if r >= 2:
                        for k, v in ev.items():
                            parts_ts[B][k].append(v)
            if r >= 2:
                e2e_ts.append(row)
        torch.cuda.synchronize()
        e2e_total = torch.tensor([sum(a.elapsed_time(b) for row in e2e_ts for a, b in row)],
                                 dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
        breakdown = None
        if world == 1:
            breakdown = []
            for i, B in enumerate(batches):
                ev = lambda lst: round(float(np.mean([a.elapsed_time(b) for a, b in lst])) * 1000.0, 2)
                breakdown.append({"B": B,
                                  "e2e_us": round(float(np.mean([row[i][0].elapsed_time(row[i][1])
                                                                 for row in e2e_ts])) * 1000.0, 2),
                                  "copies_us": ev(parts_ts[B]["copies"]),
                                  "copies_dma_us": ev(parts_ts[B]["copies_dma"]),
                                  "eager_call_us": ev(parts_ts[B]["eager_call"]),
                                  "graph_call_us": round(per_b_us[B], 2),
                                  "h2d_bytes": B * H * 2 + B * K * 8, "d2h_bytes": B * H * 2})
        e2e = {"value": round(float(e2e_total.item()) * 1000.0 / (len(e2e_ts) * nB), 3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "breakdown": breakdown,
               "method": ("eager torch API (moe_ffn_3d_batched_host) per call"
                          if world == 1 and not mx else
                          "eager torch API (copy_ranges, moe_gate_up_3d_batched_mxfp8 + "
                          "moe_down_3d_batched_mxfp8, copy_ranges) per call"
                          if world == 1 else
                          "eager torch API (copy_ranges, FusedAllReduce.ffn or moe_gate_up_3d_batched + "
                          "moe_down_3d_batched_partial + all_reduce above the fused size, copy_ranges) "
                          "per call") +
                         ": x / topk_ids / topk_scale from pinned host memory in and y to pinned host "
                         "memory out by the library's copy kernel inside the timed window, L2 flushed "
                         "before each call"}

    others = None
    if world == 1 and args.workload == WORKLOAD and not args.no_extras and not args.no_others:
        others = run_other_workloads_leg(args, dev, flush, stream, cur, peak_gbs)

    tp_full = None
    if args.workload == WORKLOAD and not args.no_extras and not args.no_tp_full:
        for c in cases.values():
            del c.g_e2e, c.g_gu, c.g_dn, c.g_split, c.g_nccl
        torch.cuda.empty_cache()
        tp_full = run_tp_full_leg(args, rank, local_rank, world, dev, flush, stream, cur,
                                  fused, peak_gbs)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_timing(batches, H, I, E, K, cfg.routing, budget_s=args.cpu_seconds,
                                   steps=None)
        if mx:
            cpu["sample"] += " (bf16 weights: the reference has no MXFP8 path)"

    clocks_all = [clocks]
    if world > 1:
        clocks_all = [None] * world
        dist.all_gather_object(clocks_all, clocks)
    if rank == 0:
        mhz = [c["sm_mhz"] for c in clocks_all if c and c.get("sm_mhz")]
        reasons = sorted({r for c in clocks_all if c for r in c.get("reasons", [])})
        clock_rec = {"sm_mhz": statistics.median(mhz) if mhz else None,
                     "sm_max_mhz": clocks_all[0].get("sm_max_mhz") if clocks_all[0] else None,
                     "reasons": reasons, "samples": sum(c.get("samples", 0) for c in clocks_all if c)}
        wname = workload_name(args.workload, cfg, world)
        routing = {"uniform": "uniform distinct", "zipf": "Zipf(1.1) distinct"}.get(cfg.routing, cfg.routing)
        line = {
            "metric": METRIC, "value": round(value_us, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": False, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "e4m3 weights (MXFP8, ue8m0 per 32) x bf16 activations, fp32 accumulate" if mx else "bf16",
            "data": f"synthetic (seeded; x~N(0,1), W~N(0,fan_in^-1/2), {routing} top-{K}, softmax weights"
                    + (", W quantised to MXFP8 on the device)" if mx else ")"),
            "config": {"workload": wname,
                       "hidden": H, "inter_per_gpu": I, "inter_total": cfg.inter_full if strong else I * world, "experts": E,
                       "topk": K, "batches": batches, "global_batch": batches,
                       "parallelism": "single GPU" if world == 1 else (
                           f"tp{world} over inter + all-reduce fused into the kernels (NVLink peer stores; "
                           f"one launch for B*topk <= 32) "
                           f"for B <= {max([B for B in batches if fused.applies(B)], default=0)}, NCCL above"
                           if fused is not None else f"tp{world} over inter + NCCL all-reduce"),
                       "l2": "flushed before every timed call (256 MiB write + 256 MiB read)",
                       "timing": "CUDA graph replay per call, CUDA events on the launching stream, "
                                 "value = mean us/call over the sweep, max over ranks"},
            "impl": "ours",
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clock_rec,
            "gpu_launches": args.steps * sum(launches.values()),
            "parity": parity,
            "sweep": sweep,
            "tp_full": tp_full,
            "other_workloads": others,
        }
        print(json.dumps(line), flush=True)

    if tp_full is None:
        for c in cases.values():
            del c.g_e2e, c.g_gu, c.g_dn, c.g_split, c.g_nccl
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        if fused is not None:
            fused.close()
        dist.destroy_process_group()
    return 0


def exchange_record(fused, B, H, world):
    """NVLink bytes one rank sends in the fused exchange of a [B, H] call
    (8-byte packets: one-shot pushes every partial row to every peer;
    two-shot pushes each row to its owner and the owner's bf16 result back),
    or None where the call is not fused."""
    if world == 1 or fused is None or not fused.applies(B):
        return None
    one_shot = B * H * 8 * (world - 1)
    two_shot = world >= 4 and one_shot > int(os.environ.get("WARP_DECODE_TP_TWO_SHOT_BYTES") or 16 << 20)
    sent = 2 * B * H * 8 * (world - 1) // world if two_shot else one_shot
    return {"shape": "two-shot" if two_shot else "one-shot", "bytes_sent_per_rank": sent}


def cold_us(fn, flush, stream, cur, reps):
    """Mean cold us of fn(): CUDA graph of one call, L2 flushed before each
    replay, CUDA events around the replay only."""
    import numpy as np
    import torch

    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        out = fn()
    ts = []
    for _ in range(reps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        g.replay()
        b.record(cur)
        ts.append((a, b))
    torch.cuda.synchronize()
    del g, out
    return float(np.mean([a.elapsed_time(b) for a, b in ts]) * 1000.0)


def run_other_workloads_leg(args, dev, flush, stream, cur, peak_gbs):
    """BASELINE configs[3] (DeepSeek-V3 TP=8 shard, Zipf routing) and
    configs[4] (Qwen3-30B-A3B with MXFP8 weights, next to the same shape in
    bf16) after the headline, one GPU: cold us per call through the public
    API at each of the config's batch sizes, and the fraction of measured HBM
    on the call's algorithmic bytes.  Reported beside the headline; it does
    not change `value`."""
    import torch

    from warp_decode_b200 import warp_decode as wd
    from warp_decode_b200 import workloads as W
    from warp_decode_b200.mxfp8 import quantize_mxfp8

    reps = max(5, min(args.kernel_reps, 20))
    out = {}

    def leg(name, weights, make_call, bf16_w=None):
        cfg = W.CONFIGS[name]
        H, I, E, K = cfg.hidden, cfg.inter, cfg.E, cfg.topk
        rows = []
        for B in cfg.batches:
            x, ids, scale = W.make_device_activations(B, H, E, K, cfg.routing, args.seed + 700 + B,
                                                      device=dev)
            U = W.unique_experts(ids.cpu().numpy())
            nb = W.algorithmic_bytes(U, B, H, I, K, weights)["e2e"]
            us = cold_us(make_call(x, ids, scale), flush, stream, cur, reps)
            row = {"B": B, "us": round(us, 2), "unique_experts": U, "bytes": nb,
                   "hbm_frac": round(nb / (us * 1e-6) / 1e9 / peak_gbs, 3)}
            if bf16_w is not None:
                wgu, wdn = bf16_w
                row["bf16_us_same_shape"] = round(
                    cold_us(lambda: wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale), flush, stream,
                            cur, reps), 2)
            rows.append(row)
        return {"config": name, "hidden": H, "inter": I, "experts": E, "topk": K,
                "routing": cfg.routing, "weights": weights, "unit": UNIT,
                "timing": f"cold (L2 flushed), CUDA graph replay, CUDA events, mean of {reps} calls",
                "per_batch": rows}

    c = W.CONFIGS["dsv3_tp8"]
    wgu, wdn = W.make_device_weights(c.hidden, c.inter, c.E, args.seed + 3, device=dev)
    out["dsv3_tp8"] = leg("dsv3_tp8", "bf16", lambda x, ids, sc: (
        lambda: wd.moe_ffn_3d_batched(x, wgu, wdn, ids, sc)))
    del wgu, wdn
    torch.cuda.empty_cache()
    c = W.CONFIGS["qwen3_30b_mxfp8"]
    wgu, wdn = W.make_device_weights(c.hidden, c.inter, c.E, args.seed + 5, device=dev)
    gq, gs = quantize_mxfp8(wgu)
    dq, ds = quantize_mxfp8(wdn)
    out["qwen3_30b_mxfp8"] = leg("qwen3_30b_mxfp8", "mxfp8", lambda x, ids, sc: (
        lambda: wd.moe_down_3d_batched_mxfp8(wd.moe_gate_up_3d_batched_mxfp8(x, gq, gs, ids),
                                             dq, ds, ids, sc, x.shape[0])), bf16_w=(wgu, wdn))
    del wgu, wdn, gq, gs, dq, ds
    torch.cuda.empty_cache()
    return out


def run_tp_full_leg(args, rank, local_rank, world, dev, flush, stream, cur, fused, peak_gbs):
    """BASELINE configs[2] after the headline: the full-width Qwen3-235B FFN
    (hidden 4096, inter 1536, 128 experts, top-8) split over the N GPUs
    (inter 1536 / N per GPU: TP1/2/4/8 = 1536/768/384/192), strong scaling,
    at B in {1, 4, 16, 64}: cold us per call (L2 flushed, CUDA graph, events
    on the launching stream, max over ranks) and the per-GPU HBM fraction on
    that GPU's algorithmic bytes.  Reported beside the headline; it does not
    change `value`."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from warp_decode_b200 import warp_decode as wd
    from warp_decode_b200 import workloads as W

    cfg = W.CONFIGS["qwen3_235b_full"]
    H, E, K = cfg.hidden, cfg.E, cfg.topk
    I = cfg.inter_full // world
    w_gu, w_dn = W.make_device_weights(H, I, E, args.seed + 31 + 7919 * rank, device=dev)
    reps = max(5, min(args.kernel_reps, 20))
    rows = []
    for B in cfg.batches:
        x, ids, scale = W.make_device_activations(B, H, E, K, cfg.routing, args.seed + 500 + B,
                                                  device=dev)
        U = W.unique_experts(ids.cpu().numpy())
        nbytes = W.algorithmic_bytes(U, B, H, I, K)["e2e"]

        def call():
            if world == 1:
                return wd.moe_ffn_3d_batched(x, w_gu, w_dn, ids, scale)
            if fused is not None and fused.applies(B):
                return fused.ffn(x, w_gu, w_dn, ids, scale)
            h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
            part = wd.moe_down_3d_batched_partial(h, w_dn, ids, scale, B)
            dist.all_reduce(part)
            return part.to(torch.bfloat16)

        with torch.cuda.stream(stream):
            for _ in range(3):
                call()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            call()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        ts = []
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            g.replay()
            b.record(cur)
            ts.append((a, b))
        torch.cuda.synchronize()
        us = torch.tensor([float(np.mean([a.elapsed_time(b) for a, b in ts]) * 1000.0)],
                          dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
        us = float(us.item())
        rows.append({"B": B, "us": round(us, 2), "unique_experts": U,
                     "bytes_per_gpu": nbytes,
                     "hbm_frac_per_gpu": round(nbytes / (us * 1e-6) / 1e9 / peak_gbs, 3)})
        del g
        torch.cuda.synchronize()
    del w_gu, w_dn
    torch.cuda.empty_cache()
    return {"workload": f"qwen3_235b_full_tp{world}", "config": "BASELINE configs[2]",
            "hidden": H, "inter_total": cfg.inter_full, "inter_per_gpu": I, "experts": E,
            "topk": K, "scaling": "strong", "unit": UNIT,
            "timing": "cold (L2 flushed), CUDA graph replay, CUDA events, mean of "
                      f"{reps} calls, max over ranks",
            "per_batch": rows, "mean_us": round(sum(r["us"] for r in rows) / len(rows), 3)}


# ---------------------------------------------------------------------------
# CPU (reference PyTorch path) timing
# ---------------------------------------------------------------------------
def cpu_reference_timing(batches, H, I, E, K, routing, budget_s=12.0, steps=None, warmup=0,
                         seed=99):
    """Time oracle.torch_port (the reference's gather + bmm path) on the host cores.

    Bounded sample: each call runs on at most `cap` tokens of its batch (the
    reference path is linear in the routed slots), with `cap` chosen so the
    whole run stays inside `budget_s`; the time is scaled by B / tokens.
    Returns per-batch us/call and the sweep mean.
    """
    import numpy as np
    import torch

    from oracle import torch_port as P
    from warp_decode_b200 import workloads as W

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rng = np.random.default_rng(seed)

    def make(Bs):
        ids = W.host_routing(rng, Bs, E, K, routing, seed)
        uniq, inv = np.unique(ids, return_inverse=True)
        n = len(uniq)  # compact tensor with just the touched experts
        g = torch.Generator().manual_seed(int(rng.integers(1 << 30)))
        w_gu = (torch.randn(n, 2 * I, H, generator=g) * H ** -0.5).bfloat16()
        w_dn = (torch.randn(n, H, I, generator=g) * I ** -0.5).bfloat16()
        x = torch.randn(Bs, H, generator=g).bfloat16()
        sc = torch.softmax(torch.randn(Bs, K, generator=g), dim=1)
        return x, w_gu, w_dn, torch.from_numpy(inv.reshape(Bs, K).astype(np.int32)), sc

    # calibrate one token's cost
    x, wg, wdn, ids, sc = make(1)
    P.moe_ffn(x, wg, wdn, ids, sc)
    t0 = time.perf_counter()
    P.moe_ffn(x, wg, wdn, ids, sc)
    per_tok = max(time.perf_counter() - t0, 1e-6)
    nsteps = steps if steps is not None else 3
    total_calls = (nsteps + warmup) * len(batches)
    cap = max(1, int(budget_s / (total_calls * per_tok)))
    per_b = {}
    inputs = {B: make(min(B, cap)) for B in batches}
    step_ms = []
    for s in range(warmup + nsteps):
        tot = 0.0
        for B in batches:
            x, wg, wdn, ids, sc = inputs[B]
            t0 = time.perf_counter()
            P.moe_ffn(x, wg, wdn, ids, sc)
            dt = (time.perf_counter() - t0) * B / x.shape[0]
            if s >= warmup:
                per_b.setdefault(B, []).append(dt)
            tot += dt
        if s >= warmup:
            step_ms.append(tot * 1000.0)
    per_b_us = {B: statistics.median(v) * 1e6 for B, v in per_b.items()}
    mean_us = sum(per_b_us.values()) / len(per_b_us)
    return {"value": round(mean_us, 1), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle/torch_port.py (reference gather+bf16 bmm path) on CPU, {threads} threads, "
                      f"{nsteps} sweeps, each call on min(B, {cap}) tokens scaled by B/tokens",
            "per_batch_us": {str(B): round(v, 1) for B, v in per_b_us.items()},
            "step_ms": step_ms}


def workload_name(workload, cfg, world):
    """config.workload of the JSON line for `workload` run on `world` GPUs."""
    if world == 1:
        return workload
    if workload == "qwen3_235b_full":
        return f"{workload}_tp{world}"
    if workload == WORKLOAD:
        return f"qwen3_235b_inter{cfg.inter * world}_tp{world}"
    return f"{workload}_inter{cfg.inter * world}_tp{world}"


def run_reference(args, rank, world):
    """--impl reference: the reference's PyTorch path on the host cores (rank 0 only)."""
    if rank != 0:
        return 0
    from warp_decode_b200 import workloads as W

    cfg = W.CONFIGS[args.workload]
    batches = [int(b) for b in args.batches.split(",")] if args.batches else list(cfg.batches)
    # the reference has no tensor parallelism: the whole FFN of the N-GPU run on CPU
    I_total = cfg.inter_full if args.workload == "qwen3_235b_full" else cfg.inter * world
    budget = min(150.0, 2.0 * (args.steps + args.warmup))
    r = cpu_reference_timing(batches, cfg.hidden, I_total, cfg.E, cfg.topk, cfg.routing,
                             budget_s=budget, steps=args.steps, warmup=args.warmup)
    ms_per_step = statistics.mean(r["step_ms"])
    line = {
        "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": False,
        "scaling": "strong" if args.workload == "qwen3_235b_full" else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload_name(args.workload, cfg, world),
                   "hidden": cfg.hidden, "inter_total": I_total, "experts": cfg.E, "topk": cfg.topk,
                   "batches": batches, "parallelism": "CPU, all host threads"},
        "impl": "reference",
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "per_batch_us": r["per_batch_us"],
        "reference_gpu_kernels": (reference_gpu_kernels_leg(args, batches)
                                  if world == 1 and args.workload == WORKLOAD else None),
    }
    print(json.dumps(line), flush=True)
    return 0


def reference_gpu_kernels_leg(args, batches):
    """The reference's own CUDA kernels (csrc/*.cu, rebuilt unmodified for
    sm_100a into oracle/_ref/ by oracle/Makefile) on this GPU, by the method
    of the headline: gate_up + down of each batch size in one CUDA graph, L2
    flushed before each replay, CUDA events around the replay, the headline's
    inputs (same seeds); beside them this library's e2e call timed the same
    way.  A same-box GPU bar for the headline, reported with the reference
    arm; None where no GPU or no rebuilt library is present."""
    import ctypes

    try:
        import torch
    except Exception:
        return None
    lib_path = ROOT / "oracle" / "_ref" / "libwdref.so"
    if not torch.cuda.is_available() or not lib_path.exists():
        return None
    from warp_decode_b200 import warp_decode as wd
    from warp_decode_b200 import workloads as W

    L = ctypes.CDLL(str(lib_path))
    P, I_ = ctypes.c_void_p, ctypes.c_int
    L.wdref_gate_up.argtypes = [P, P, P, P, I_, I_, I_, I_, I_, P]
    L.wdref_down.argtypes = [P, P, P, P, P, I_, I_, I_, I_, I_, P]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = W.CONFIGS[WORKLOAD]
    H, I, E, K = cfg.hidden, cfg.inter, cfg.E, cfg.topk
    w_gu, w_dn = W.make_device_weights(H, I, E, args.seed, device=dev)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream(dev)
    reps = max(5, min(args.kernel_reps, 20))
    rows = []
    for B in batches:
        x, ids, scale = W.make_device_activations(B, H, E, K, cfg.routing, args.seed + B, device=dev)
        h = torch.empty(B * K, I, dtype=torch.bfloat16, device=dev)
        y = torch.empty(B, H, dtype=torch.bfloat16, device=dev)

        def ref_e2e():
            st = torch.cuda.current_stream().cuda_stream
            L.wdref_gate_up(x.data_ptr(), w_gu.data_ptr(), ids.data_ptr(), h.data_ptr(), B, E, K,
                            H, I, st)
            L.wdref_down(h.data_ptr(), w_dn.data_ptr(), ids.data_ptr(), scale.data_ptr(),
                         y.data_ptr(), B, E, K, H, I, st)

        ref = cold_us(ref_e2e, flush, stream, cur, reps)
        ours = cold_us(lambda: wd.moe_ffn_3d_batched(x, w_gu, w_dn, ids, scale), flush, stream,
                       cur, reps)
        rows.append({"B": B, "reference_kernels_us": round(ref, 2), "ours_us": round(ours, 2),
                     "speedup": round(ref / ours, 2)})
    del w_gu, w_dn
    torch.cuda.empty_cache()
    return {"what": "csrc/moe_gate_up_3d_batched.cu + csrc/moe_down_3d_batched.cu of the "
                    "reference, compiled unmodified for sm_100a, two launches per call",
            "timing": f"cold (L2 flushed), CUDA graph replay, CUDA events, mean of {reps} calls",
            "unit": UNIT, "per_batch": rows,
            "mean_reference_kernels_us": round(sum(r["reference_kernels_us"] for r in rows) / len(rows), 3),
            "mean_ours_us": round(sum(r["ours_us"] for r in rows) / len(rows), 3)}


def main():
    args = parse_args()
    rank, local_rank, world = env_rank()
    if world != args.gpus and args.gpus > 1 and world == 1:
        print(f"--gpus {args.gpus} needs torchrun with {args.gpus} processes", file=sys.stderr)
        return 2
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
