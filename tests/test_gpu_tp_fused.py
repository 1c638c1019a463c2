"""Tensor-parallel FFN with the all-reduce fused into the kernels.

Two processes on two GPUs (skipped with fewer): each rank holds half of the
intermediate dimension of a Qwen3-235B-style FFN; the fused path
(FusedAllReduce: epoch-tagged packets pushed to every rank by the single-launch
FFN kernel at small B, by the tcgen05 down kernel above) must match the NCCL
path and the unsharded FP32 oracle (rtol = atol = 1e-2), give
bitwise-identical outputs on both ranks and in both exchange shapes
(one-shot and two-shot), keep its epochs in step when the two
kernels take turns on one communicator, survive CUDA-graph replay (epochs
advance), and end a wait whose peer never arrives with WD_STATUS_WAIT_TIMEOUT
within the 2 s bound instead of hanging.  NVLS is off (NCCL_NVLS_ENABLE=0).
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import moe_ref as O
    from warp_decode_b200 import workloads as W
    from warp_decode_b200.tp import FusedAllReduce, TensorParallelMoE

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, device_id=dev, timeout=timedelta(seconds=60))
    H, I, E, K = 4096, 384, 128, 8  # two ranks x 192
    w_gu, w_dn = W.make_device_weights(H, I, E, 77, device=dev)
    fused = FusedAllReduce(H, max_tokens=64)
    moe_nccl = TensorParallelMoE(w_gu, w_dn)
    moe_fused = TensorParallelMoE(w_gu, w_dn, fused=fused)
    res = {}
    from warp_decode_b200 import warp_decode as wd
    for B in (1, 8, 64):
        dist.barrier(device_ids=[rank])
        x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 900 + B, device=dev)
        y_nccl = moe_nccl(x, ids, scale)
        y_fused = moe_fused(x, ids, scale)
        torch.cuda.synchronize()
        res[f"status_{B}"] = wd.status(True, rank)
        res[f"fused_{B}"] = y_fused.cpu().view(torch.int16).numpy()
        res[f"nccl_{B}"] = y_nccl.cpu().view(torch.int16).numpy()
        if rank == 0:
            ids_h = ids.cpu().numpy()
            touched = lambda w: {int(e): w[int(e)].cpu().view(torch.int16).numpy().view(np.uint16)
                                 for e in np.unique(ids_h)}
            xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
            h_ref = O.gate_up(xb, touched(w_gu), ids_h)
            res[f"ref_{B}"] = O.down(h_ref, touched(w_dn), ids_h, scale.cpu().numpy())
    # Both exchange shapes, forced, on both kernels: the same bits.
    for mode in (1, 2):
        fused.set_exchange(mode)
        for B in (1, 8, 64):
            dist.barrier(device_ids=[rank])
            x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 900 + B, device=dev)
            y = moe_fused(x, ids, scale)
            torch.cuda.synchronize()
            res[f"mode{mode}_{B}"] = y.cpu().view(torch.int16).numpy()
            res[f"mode{mode}_status_{B}"] = wd.status(True, rank)
    fused.set_exchange(0)
    # The single-launch FFN (B = 1) and the tcgen05 down kernel (B = 4) take
    # turns on one communicator: every call advances every epoch entry.  The
    # ranks enter every fused call within the 2 s wait bound of each other
    # (rank 0 just spent seconds on the CPU oracle): barrier first.
    dist.barrier(device_ids=[rank])
    xa, ida, sca = W.make_device_activations(1, H, E, K, "uniform", 2101, device=dev)
    xb, idb, scb = W.make_device_activations(4, H, E, K, "uniform", 2104, device=dev)
    alt_a, alt_b = [], []
    for _ in range(3):
        alt_a.append(fused.ffn(xa, moe_fused.w_gu, moe_fused.w_dn, ida, sca))
        hb = wd.moe_gate_up_3d_batched(xb, moe_fused.w_gu, idb)
        alt_b.append(fused.down(hb, moe_fused.w_dn, idb, scb))
    ya_n, yb_n = moe_nccl(xa, ida, sca), moe_nccl(xb, idb, scb)
    torch.cuda.synchronize()
    res["alt_status"] = wd.status(True, rank)
    res["alt_a"] = np.stack([t.cpu().view(torch.int16).numpy() for t in alt_a])
    res["alt_b"] = np.stack([t.cpu().view(torch.int16).numpy() for t in alt_b])
    res["alt_a_nccl"] = ya_n.cpu().view(torch.int16).numpy()
    res["alt_b_nccl"] = yb_n.cpu().view(torch.int16).numpy()
    # graph replay (single launch at B = 2, two kernels at B = 16): epochs
    # advance inside the graph.
    for B in (2, 16):
        dist.barrier(device_ids=[rank])
        x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 1900 + B, device=dev)
        s = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(s):
            for _ in range(2):
                moe_fused(x, ids, scale)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y_g = moe_fused(x, ids, scale)
        outs = []
        for _ in range(5):
            g.replay()
            torch.cuda.synchronize()
            outs.append(y_g.cpu().view(torch.int16).numpy().copy())
        dist.barrier(device_ids=[rank])
        res[f"graph_{B}"] = np.stack(outs)
        res[f"graph_eager_{B}"] = moe_fused(x, ids, scale).cpu().view(torch.int16).numpy()
        res[f"graph_status_{B}"] = wd.status(True, rank)
        del g
    dist.barrier(device_ids=[rank])
    # a peer that never arrives: only rank 0 calls the fused down
    if rank == 0:
        import time

        h = torch.zeros(B * K, I // WORLD, dtype=torch.bfloat16, device=dev)
        t0 = time.time()
        y = fused.down(h, moe_fused.w_dn, ids, scale)
        torch.cuda.synchronize()
        res["timeout_s"] = time.time() - t0
        res["timeout_status"] = wd.status(True, rank)
        res["timeout_out_zero"] = bool((y.float() == 0).all().item())
    dist.barrier(device_ids=[rank])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    # the abandoned call left this rank one epoch ahead: drop the communicator
    fused.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
def test_fused_allreduce_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    from conftest import bf16_close

    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    r0 = dict(np.load(tmp_path / "rank0.npz"))
    r1 = dict(np.load(tmp_path / "rank1.npz"))
    for B in (1, 8, 64):
        assert r0[f"status_{B}"] == 0 and r1[f"status_{B}"] == 0
        f0, f1 = r0[f"fused_{B}"].view(np.uint16), r1[f"fused_{B}"].view(np.uint16)
        assert np.array_equal(f0, f1), "fused all-reduce must give identical bits on all ranks"
        ok, d = bf16_close(f0, r0[f"ref_{B}"], 1e-2, 1e-2)
        assert ok, f"B={B}: fused vs oracle max |diff| {d}"
        ok, d = bf16_close(r0[f"nccl_{B}"].view(np.uint16), r0[f"ref_{B}"], 1e-2, 1e-2)
        assert ok, f"B={B}: NCCL path vs oracle max |diff| {d}"
        for r in (r0, r1):
            for mode in (1, 2):
                assert r[f"mode{mode}_status_{B}"] == 0
                assert np.array_equal(r[f"mode{mode}_{B}"].view(np.uint16), f0), \
                    f"B={B}: exchange shape {mode} changed the bits"
    for r in (r0, r1):
        for B in (2, 16):
            g = r[f"graph_{B}"]
            assert r[f"graph_status_{B}"] == 0
            assert all(np.array_equal(g[0], g[i]) for i in range(1, len(g)))
            assert np.array_equal(g[0], r[f"graph_eager_{B}"])
        assert r["alt_status"] == 0
        for key in ("alt_a", "alt_b"):
            a = r[key].view(np.uint16)
            assert all(np.array_equal(a[0], a[i]) for i in range(1, len(a)))
            ok, d = bf16_close(a[0], r[key + "_nccl"].view(np.uint16), 1e-2, 1e-2)
            assert ok, f"{key}: fused vs NCCL max |diff| {d}"
    assert np.array_equal(r0["alt_a"], r1["alt_a"]) and np.array_equal(r0["alt_b"], r1["alt_b"])
    assert r0["timeout_status"] & 0x2, "a missing peer must end in WD_STATUS_WAIT_TIMEOUT"
    assert r0["timeout_s"] < 30.0
    assert r0["timeout_out_zero"]
