"""CPU oracle for the fused MoE decode path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The CUDA path in ``warp_decode_b200`` never calls it.

It restates, in numpy, the reference's PyTorch path (Religious-J/warp_decode):

* ``gate_up(..., mode="bf16")``  -- ``reference_gate_up``,
  tests/test_gate_up_correctness.py:19-43: gather W[ids], bf16 bmm with the
  result rounded to bf16, ``silu(gate) * up`` in bf16 arithmetic.
* ``down(..., mode="bf16")``     -- ``reference_down``,
  tests/test_down_correctness.py:14-35: gather W[ids], bf16 bmm rounded to
  bf16, then ``.float() * topk_scale`` and an FP32 sum over the top-k slots.
* ``gate_up/down(..., mode="fp32")`` -- the FP32-accumulated reference the
  kernels are held to, tests/test_benchmark_reference.py:36-43: operands
  upcast to FP32, ``silu(gate) * up`` in FP32 rounded to bf16 (the bf16
  boundary at the activation buffer), down projection in FP32, scaled and
  summed over slots in FP32, rounded to bf16 once.

Dot products are evaluated in float64 and rounded to float32, i.e. the exact
FP32 value of each projection (the reference's bmm accumulates in FP32 in an
unspecified order; the difference is far below the bf16 output resolution).

It also restates the OCP Microscaling Formats (MX) v1.0 MXFP8-E4M3 encoding
(shared exponent = floor(log2(amax)) - 8 per block of 32 along the reduction
axis, elements rounded to nearest-even E4M3 with saturation at 448, scale
stored as a biased ue8m0 byte), which the reference lists as future work
(README.md:294-308) and which therefore has no reference source to follow.

The router producer (``router_topk``) has no reference source either (the
reference takes topk_ids / topk_scale as inputs); it restates the usual MoE
router: top-k of the logits (softmax is monotonic), weights = softmax over
the selected logits when renormalised, else softmax over all logits at the
selected ids.  Its parity is "unpinned" against the reference (nothing to
pin to) and checked against torch.topk / torch.softmax in the tests.

Parity pins: ``tests/golden/`` holds outputs of the reference's own
``reference_gate_up`` / ``reference_down`` and of its FP32 formula, generated
by ``tests/golden/make_golden.py``; ``tests/test_oracle.py`` checks this module
against them.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_to_f32", "f32_to_bf16", "silu_f32", "gate_up", "down", "moe_ffn",
    "e4m3_to_f32", "f32_to_e4m3", "mx_quantize", "mx_dequantize", "E4M3_MAX", "router_topk",
]

E4M3_MAX = 448.0


# ---------------------------------------------------------------------------
# bf16 helpers (bf16 stored as uint16 bit patterns)
# ---------------------------------------------------------------------------
def bf16_to_f32(u16) -> np.ndarray:
    """bf16 bit patterns -> float32 (exact: a bf16 is the top half of an fp32)."""
    u16 = np.asarray(u16, dtype=np.uint16)
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN stays NaN)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


def _round_bf16(f) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(f))


def silu_f32(v) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


def _expert_rows(w, e):
    """w is a [E, ...] array or a mapping expert -> [...] array (touched experts only)."""
    return np.asarray(w[int(e)])


# ---------------------------------------------------------------------------
# gate_up
# ---------------------------------------------------------------------------
def gate_up(x_u16, w_gate_up, topk_ids, mode: str = "fp32", inter: int | None = None) -> np.ndarray:
    """h[b*K+s, n] = silu(x[b].W[e,n]) * x[b].W[e,I+n], e = topk_ids[b,s]; bf16 bits out.

    x_u16     : [B, H] uint16 (bf16 bits)
    w_gate_up : [E, 2I, H] uint16, or mapping expert -> [2I, H] uint16 (or float32 for
                already-dequantised MXFP8 weights)
    topk_ids  : [B, K] int
    mode      : "fp32" (tests/test_benchmark_reference.py:36-40) or
                "bf16" (tests/test_gate_up_correctness.py:19-43)
    """
    x = bf16_to_f32(x_u16).astype(np.float64)
    ids = np.asarray(topk_ids)
    B, K = ids.shape
    out = None
    flat = ids.reshape(-1)
    for e in np.unique(flat):
        slots = np.nonzero(flat == e)[0]
        wr = _expert_rows(w_gate_up, e)
        wf = (bf16_to_f32(wr) if wr.dtype == np.uint16 else wr.astype(np.float32)).astype(np.float64)
        two_i = wf.shape[0]
        I = two_i // 2 if inter is None else inter
        if out is None:
            out = np.zeros((B * K, I), dtype=np.uint16)
        proj = (x[slots // K] @ wf.T).astype(np.float32)  # [n_slots, 2I] exact-then-fp32
        g, u = proj[:, :I], proj[:, I:]
        if mode == "fp32":
            h = f32_to_bf16(silu_f32(g) * u)
        elif mode == "bf16":
            gb, ub = _round_bf16(g), _round_bf16(u)
            s = _round_bf16(silu_f32(gb))
            h = f32_to_bf16(s * ub)
        else:
            raise ValueError(mode)
        out[slots] = h
    if out is None:
        raise ValueError("empty routing")
    return out


# ---------------------------------------------------------------------------
# down
# ---------------------------------------------------------------------------
def down(h_u16, w_down, topk_ids, topk_scale, mode: str = "fp32", return_f32: bool = False):
    """y[b, j] = sum_s scale[b,s] * h[b*K+s].Wd[e_s, j]; bf16 bits out (or fp32 pre-rounding).

    h_u16      : [B*K, I] uint16
    w_down     : [E, H, I] uint16, or mapping expert -> [H, I]
    topk_scale : [B, K] float32
    mode       : "fp32" (tests/test_benchmark_reference.py:41-43) or
                 "bf16" (tests/test_down_correctness.py:14-35)
    """
    hh = bf16_to_f32(h_u16).astype(np.float64)
    ids = np.asarray(topk_ids)
    scale = np.asarray(topk_scale, dtype=np.float32)
    B, K = ids.shape
    flat = ids.reshape(-1)
    proj = None
    for e in np.unique(flat):
        slots = np.nonzero(flat == e)[0]
        wr = _expert_rows(w_down, e)
        wf = (bf16_to_f32(wr) if wr.dtype == np.uint16 else wr.astype(np.float32)).astype(np.float64)
        if proj is None:
            proj = np.zeros((B * K, wf.shape[0]), dtype=np.float32)
        p = (hh[slots] @ wf.T).astype(np.float32)  # [n_slots, H]
        proj[slots] = _round_bf16(p) if mode == "bf16" else p
    if proj is None:
        raise ValueError("empty routing")
    if mode not in ("fp32", "bf16"):
        raise ValueError(mode)
    H = proj.shape[1]
    scaled = proj.reshape(B, K, H) * scale[:, :, None]
    y = np.zeros((B, H), dtype=np.float32)
    for s in range(K):  # FP32 sum over the slots
        y = (y + scaled[:, s, :]).astype(np.float32)
    return y if return_f32 else f32_to_bf16(y)


def moe_ffn(x_u16, w_gate_up, w_down, topk_ids, topk_scale, mode: str = "fp32"):
    """End-to-end MoE FFN: down(gate_up(x)) with the bf16 boundary at h."""
    h = gate_up(x_u16, w_gate_up, topk_ids, mode=mode)
    return down(h, w_down, topk_ids, topk_scale, mode=mode)


# ---------------------------------------------------------------------------
# OCP MX v1.0 -- MXFP8 (E4M3 elements, E8M0 shared scale, block 32)
# ---------------------------------------------------------------------------
def _e4m3_table() -> np.ndarray:
    codes = np.arange(0x7F, dtype=np.int64)  # 0x00..0x7E: non-negative finite values
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    val = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp - 7.0))
    return val.astype(np.float64)


_E4M3_VALUES = _e4m3_table()


def e4m3_to_f32(q) -> np.ndarray:
    """E4M3 (OCP 'fn': no inf, S.1111.111 = NaN) bit patterns -> float32."""
    q = np.asarray(q, dtype=np.uint8)
    mag = q & 0x7F
    val = np.where(mag == 0x7F, np.nan, _E4M3_VALUES[np.minimum(mag, 0x7E)])
    return np.where(q & 0x80, -val, val).astype(np.float32)


def f32_to_e4m3(v) -> np.ndarray:
    """float -> E4M3 bit patterns: round to nearest, ties to even mantissa, saturate at 448."""
    v = np.asarray(v, dtype=np.float64)
    a = np.minimum(np.abs(v), E4M3_MAX)
    hi = np.clip(np.searchsorted(_E4M3_VALUES, a, side="left"), 0, 0x7E)
    lo = np.clip(hi - 1, 0, 0x7E)
    d_hi = _E4M3_VALUES[hi] - a
    d_lo = a - _E4M3_VALUES[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return np.where(np.signbit(v), code | 0x80, code).astype(np.uint8)


def mx_quantize(w, block: int = 32):
    """Quantise along the last axis: returns (q uint8 [..., K], scale uint8 [..., K/32])."""
    w = np.asarray(w, dtype=np.float32)
    K = w.shape[-1]
    if K % block:
        raise ValueError("last axis must be a multiple of the block size")
    blocks = w.reshape(*w.shape[:-1], K // block, block).astype(np.float64)
    amax = np.abs(blocks).max(axis=-1)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(amax > 0, amax, 1.0))) - 8.0  # emax(E4M3) = 8
    e = np.where(amax > 0, e, -127.0)
    e = np.clip(e, -127.0, 127.0)
    q = f32_to_e4m3(blocks / np.exp2(e)[..., None])
    return q.reshape(w.shape), (e + 127).astype(np.uint8)


def mx_dequantize(q, scale, block: int = 32) -> np.ndarray:
    """E4M3 elements times 2^(scale-127) per block of 32 along the last axis."""
    q = np.asarray(q, dtype=np.uint8)
    K = q.shape[-1]
    vals = e4m3_to_f32(q).reshape(*q.shape[:-1], K // block, block).astype(np.float64)
    s = np.exp2(np.asarray(scale, dtype=np.float64) - 127.0)
    return (vals * s[..., None]).reshape(q.shape).astype(np.float32)


# ---------------------------------------------------------------------------
# router producer (top-k + softmax)
# ---------------------------------------------------------------------------
def router_topk(logits, topk: int, renormalize: bool = True):
    """(ids int32 [B, k], weights float32 [B, k]) from logits [B, E] (float32 values).

    Order: descending logit, equal logits by ascending expert id; NaN ranks
    below every number.  Weights: exp(l - l_max) / sum, the sum over the k
    selected (renormalize) or over all E; float64 arithmetic, float32 result.
    """
    lg = np.asarray(logits, dtype=np.float64)
    lg = np.where(np.isnan(lg), -np.inf, lg)
    B, E = lg.shape
    ids = np.zeros((B, topk), dtype=np.int32)
    w = np.zeros((B, topk), dtype=np.float32)
    for b in range(B):
        order = sorted(range(E), key=lambda e: (-lg[b, e], e))[:topk]
        ids[b] = order
        sel = lg[b, order]
        ref = sel[0] if np.isfinite(sel[0]) else 0.0
        num = np.exp(sel - ref)
        den = num.sum() if renormalize else np.exp(lg[b] - ref).sum()
        w[b] = (num / den) if den > 0 else np.full(topk, 1.0 / topk)
    return ids, w
