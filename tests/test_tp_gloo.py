"""Tensor-parallel host logic on CPU ranks (gloo, world size 2 and 4).

Each rank shards the full weights with warp_decode_b200.tp, computes its FP32
partial with the CPU oracle standing in for the CUDA kernels (test-only
injection), and the ranks all-reduce over gloo.  The result must equal the
unsharded oracle FFN.  Also: a rank that never joins makes the others fail
with a timeout instead of hanging.
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleKernels:
    """CPU stand-in for the CUDA kernels (bf16 <-> uint16 bits through the oracle)."""

    @staticmethod
    def _bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    @staticmethod
    def _bf16(u16):
        return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)

    def gate_up(self, x, w, ids, w_scale=None):
        from oracle import moe_ref as O

        return self._bf16(O.gate_up(self._bits(x), self._bits(w), ids.numpy()))

    def down_partial(self, h, w, ids, scale, B, w_scale=None):
        from oracle import moe_ref as O

        return torch.from_numpy(O.down(self._bits(h), self._bits(w), ids.numpy(), scale.numpy(),
                                       return_f32=True))


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from warp_decode_b200.tp import TensorParallelMoE
    from warp_decode_b200.workloads import make_host_inputs

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        inp = make_host_inputs(3, 256, 64, 8, 4, seed=21, full=True)
        to_t = OracleKernels._bf16
        moe = TensorParallelMoE(to_t(inp["w_gate_up"]), to_t(inp["w_down"]), kernels=OracleKernels())
        assert moe.inter_local == 64 // world
        y = moe(to_t(inp["x"]), torch.from_numpy(inp["topk_ids"]), torch.from_numpy(inp["topk_scale"]))
        q.put((rank, OracleKernels._bits(y).copy()))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_matches_unsharded(world):
    from conftest import bf16_close
    from oracle import moe_ref as O
    from warp_decode_b200.workloads import make_host_inputs

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    inp = make_host_inputs(3, 256, 64, 8, 4, seed=21, full=True)
    ref = O.moe_ffn(inp["x"], inp["w_gate_up"], inp["w_down"], inp["topk_ids"], inp["topk_scale"])
    for r in range(world):
        assert not isinstance(results[r], str), results[r]
        ok, dmax = bf16_close(results[r], ref, 1e-2, 1e-2)
        assert ok, dmax
        assert np.array_equal(results[r], results[0])  # every rank holds the same output


def test_shard_layout():
    from warp_decode_b200.tp import shard_cols_down, shard_rows_gate_up

    E, I, H = 2, 8, 4
    w = torch.arange(E * 2 * I * H).reshape(E, 2 * I, H)
    s1 = shard_rows_gate_up(w, 1, 2)
    assert s1.shape == (E, I, H)
    assert torch.equal(s1[:, :4], w[:, 4:8]) and torch.equal(s1[:, 4:], w[:, 12:16])
    wd = torch.arange(E * H * I).reshape(E, H, I)
    assert torch.equal(shard_cols_down(wd, 1, 4), wd[..., 2:4])
    with pytest.raises(ValueError):
        shard_rows_gate_up(w, 0, 3)


def _absent_peer_worker(port, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=2,
                                timeout=timedelta(seconds=3))
        q.put("joined")
    except Exception as e:
        q.put(type(e).__name__)


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_absent_peer_worker, args=(_free_port(), q))
    p.start()
    out = q.get(timeout=90)
    p.join(timeout=30)
    assert out != "joined"


class _FakeCapi:
    """Records what FusedAllReduce asks of the C ABI (no GPU)."""

    def __init__(self):
        self.calls = []

    def tp_comm_create(self, world, rank, max_tokens, hidden):
        self.calls.append(("create", world, rank, max_tokens, hidden))
        return 1000 + rank, bytes([rank]) * 64

    def tp_comm_open(self, comm, handles):
        self.calls.append(("open", comm, handles))

    def torch_down_allreduce(self, h, w, ids, scale, comm):
        self.calls.append(("down", comm))
        return "y"

    def tp_comm_destroy(self, comm):
        self.calls.append(("destroy", comm))


def _fused_worker(rank, world, port, q):
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from warp_decode_b200.tp import FusedAllReduce

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=30))
    fake = _FakeCapi()
    f = FusedAllReduce(4096, max_tokens=32, _capi=fake)
    out = f.down(None, None, None, None)
    f.close()
    f.close()  # idempotent
    dist.destroy_process_group()
    q.put((rank, fake.calls, out))


@pytest.mark.parametrize("world", [2, 4])
def test_fused_allreduce_handle_exchange(world):
    """Every rank creates its communicator, opens all ranks' IPC handles in
    rank order, calls the fused down with its own communicator and destroys
    it once."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (c, o)) for r, c, o in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
    expected_handles = b"".join(bytes([r]) * 64 for r in range(world))
    for r in range(world):
        calls, out = res[r]
        assert calls[0] == ("create", world, r, 32, 4096)
        assert calls[1] == ("open", 1000 + r, expected_handles)
        assert calls[2] == ("down", 1000 + r)
        assert calls[3:] == [("destroy", 1000 + r)]
        assert out == "y"
