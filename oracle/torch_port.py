"""PyTorch-CPU port of the reference's own path -- TEST / BASELINE ONLY.

Used by bench.py's CPU baseline and ``--impl reference`` arm, which time "the
reference's PyTorch CPU path on the box's host cores" (the reference itself
cannot be imported on the GPU box).  Same algorithm as
``reference_gate_up`` (tests/test_gate_up_correctness.py:19-43) and
``reference_down`` (tests/test_down_correctness.py:14-35) of
Religious-J/warp_decode: gather every slot's expert weights, batched bf16
GEMV with torch.bmm, silu(gate)*up; down: gather, bmm, scale in FP32, sum
over the slots.  The gather materialises B*topk expert copies, so the cost is
linear in the number of routed slots.
"""
from __future__ import annotations

import torch


def gate_up(x: torch.Tensor, w: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    B, H = x.shape
    I = w.shape[1] // 2
    K = topk_ids.shape[1]
    w_sel = w.index_select(0, topk_ids.reshape(-1).long())            # [B*K, 2I, H]
    x_rep = x[:, None, :].expand(B, K, H).reshape(B * K, H, 1)
    proj = torch.bmm(w_sel, x_rep)[..., 0]                              # [B*K, 2I] bf16
    return (torch.nn.functional.silu(proj[:, :I]) * proj[:, I:]).to(torch.bfloat16)


def down(h: torch.Tensor, w: torch.Tensor, topk_ids: torch.Tensor,
         topk_scale: torch.Tensor) -> torch.Tensor:
    B, K = topk_ids.shape
    H = w.shape[1]
    w_sel = w.index_select(0, topk_ids.reshape(-1).long())            # [B*K, H, I]
    proj = torch.bmm(w_sel, h[:, :, None])[..., 0].view(B, K, H).float()
    return (proj * topk_scale[:, :, None]).sum(dim=1).to(torch.bfloat16)


def moe_ffn(x, w_gate_up, w_down, topk_ids, topk_scale):
    return down(gate_up(x, w_gate_up, topk_ids), w_down, topk_ids, topk_scale)
