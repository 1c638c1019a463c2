"""Tensor parallelism of the MoE FFN over the intermediate dimension.

The reference has no multi-GPU code ("TP" there is only a shape convention:
benchmark/bench.py:307-310 of Religious-J/warp_decode divides inter by
--tp-size).  Here the full-width FFN is split for real, one process per GPU:

* rank r of `world` keeps gate rows [r*Il, (r+1)*Il) and the matching up rows
  [I + r*Il, I + (r+1)*Il) of w_gate_up (so silu(gate)*up stays rank-local)
  and columns [r*Il, (r+1)*Il) of w_down, with Il = I / world;
* x, topk_ids and topk_scale are replicated;
* gate_up needs no communication; down produces an FP32 partial [B, hidden]
  (no bf16 rounding before the sum), followed by ONE all-reduce (NCCL over
  NVLink on GPUs) and a single bf16 rounding -- or, with FusedAllReduce, the
  down kernel itself exchanges its FP32 rows over NVLink as epoch-tagged
  8-byte packets (one-shot at small sizes, two-shot above) and sums the
  ranks' rows in rank order (one kernel, no NCCL launch, no fences).

Because silu(gate)*up is elementwise in the intermediate dimension and down
is linear in it, sum_r down_r(gate_up_r(x)) equals the unsharded FFN up to
FP32 summation order.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def shard_rows_gate_up(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[E, 2I, K] -> [E, 2*I/world, K]: this rank's gate rows then its up rows."""
    E, two_i, _ = w.shape
    inter = two_i // 2
    if inter % world:
        raise ValueError(f"inter={inter} is not divisible by world={world}")
    il = inter // world
    gate = w[:, rank * il:(rank + 1) * il]
    up = w[:, inter + rank * il: inter + (rank + 1) * il]
    return torch.cat([gate, up], dim=1).contiguous()


def shard_cols_down(w: torch.Tensor, rank: int, world: int, block: int = 1) -> torch.Tensor:
    """[E, H, I*block_factor] -> this rank's slice of the last axis.

    For MXFP8 scales of w_down pass block=32: the last axis holds I/32 scales
    and the slice is taken in units of scale blocks.
    """
    last = w.shape[-1]
    if last % world:
        raise ValueError(f"last axis {last} is not divisible by world={world}")
    n = last // world
    return w[..., rank * n:(rank + 1) * n].contiguous()


class CudaKernels:
    """The warp_decode_b200 extension (the only product implementation)."""

    def __init__(self):
        from . import warp_decode  # fails loudly if the native code is not built

        self.wd = warp_decode

    def gate_up(self, x, w, ids, w_scale=None):
        if w_scale is None:
            return self.wd.moe_gate_up_3d_batched(x, w, ids)
        return self.wd.moe_gate_up_3d_batched_mxfp8(x, w, w_scale, ids)

    def down_partial(self, h, w, ids, scale, B, w_scale=None):
        if w_scale is None:
            return self.wd.moe_down_3d_batched_partial(h, w, ids, scale, B)
        return self.wd.moe_down_3d_batched_mxfp8(h, w, w_scale, ids, scale, B, True)


class FusedAllReduce:
    """The fused all-reduce of the tensor-core down kernel for one process group.

    Collective to construct (every rank at once): each rank allocates its
    exchange buffer, the CUDA IPC handles are all-gathered over `group`, and
    every rank maps its peers' buffers.  Then ``down(h, w, ids, scale)``
    returns the bf16 sum over ranks directly (no NCCL call, no cast kernel).
    """

    def __init__(self, hidden: int, max_tokens: int = 64, group=None, _capi=None):
        if _capi is None:
            from . import capi as _capi

        capi = _capi
        self.capi = capi
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.comm, handle = capi.tp_comm_create(self.world, self.rank, max_tokens, hidden)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        capi.tp_comm_open(self.comm, b"".join(handles))

    def applies(self, B: int) -> bool:
        """Whether a call of B tokens fits the communicator (B <= max_tokens).

        The exchange shape follows the size (one-shot with two ranks and up to
        16 MiB sent per rank, two-shot above, which sends about 2/world of the
        one-shot bytes), so the fused path replaces NCCL at every batch the
        buffer holds.
        """
        return 1 <= B <= self.max_tokens

    def set_exchange(self, mode: int) -> None:
        """Force the exchange shape: 0 by size, 1 one-shot, 2 two-shot (same bits)."""
        self.capi.tp_comm_set_exchange(self.comm, mode)

    def down(self, h, w, ids, scale):
        return self.capi.torch_down_allreduce(h, w, ids, scale, self.comm)

    def ffn(self, x, w_gu, w_dn, ids, scale):
        """gate_up + down + all-reduce; one kernel launch for small batches."""
        return self.capi.torch_ffn_allreduce(x, w_gu, w_dn, ids, scale, self.comm)

    def close(self):
        if self.comm:
            self.capi.tp_comm_destroy(self.comm)
            self.comm = None


class TensorParallelMoE:
    """One rank's share of a tensor-parallel MoE FFN (decode).

    Construct on every rank with the FULL weights (or pre-sharded ones with
    ``presharded=True``); call with replicated x / topk_ids / topk_scale.
    Every rank must call with the same batch in the same order (the single
    all-reduce is a collective).
    """

    def __init__(self, w_gate_up, w_down, *, rank: Optional[int] = None,
                 world: Optional[int] = None, group=None, w_gate_up_scale=None,
                 w_down_scale=None, presharded: bool = False, kernels=None,
                 fused: Optional[FusedAllReduce] = None):
        self.group = group
        self.fused = fused
        if world is None:
            world = dist.get_world_size(group) if dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rank, self.world = rank, world
        self.kernels = kernels if kernels is not None else CudaKernels()
        if presharded or world == 1:
            self.w_gu, self.w_dn = w_gate_up, w_down
            self.s_gu, self.s_dn = w_gate_up_scale, w_down_scale
        else:
            self.w_gu = shard_rows_gate_up(w_gate_up, rank, world)
            self.w_dn = shard_cols_down(w_down, rank, world)
            self.s_gu = None if w_gate_up_scale is None else shard_rows_gate_up(w_gate_up_scale, rank, world)
            self.s_dn = None if w_down_scale is None else shard_cols_down(w_down_scale, rank, world)

    @property
    def inter_local(self) -> int:
        return self.w_gu.shape[1] // 2

    def partial(self, x, topk_ids, topk_scale):
        """This rank's FP32 contribution [B, hidden] (before the all-reduce)."""
        B = x.shape[0]
        h = self.kernels.gate_up(x, self.w_gu, topk_ids, self.s_gu)
        return self.kernels.down_partial(h, self.w_dn, topk_ids, topk_scale, B, self.s_dn)

    def __call__(self, x, topk_ids, topk_scale):
        if (self.fused is not None and self.world > 1 and self.s_dn is None
                and self.fused.applies(x.shape[0])):
            if self.s_gu is None:
                return self.fused.ffn(x, self.w_gu, self.w_dn, topk_ids, topk_scale)
            h = self.kernels.gate_up(x, self.w_gu, topk_ids, self.s_gu)
            return self.fused.down(h, self.w_dn, topk_ids, topk_scale)
        part = self.partial(x, topk_ids, topk_scale)
        if self.world > 1:
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return part.to(torch.bfloat16)
