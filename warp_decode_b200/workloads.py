"""Seeded synthetic MoE-decode workloads and the roofline byte model.

The shapes and value distributions are those of the benchmark configurations
(a Qwen3-235B TP=8 shard, the full-width Qwen3-235B FFN split tensor-parallel,
a DeepSeek-V3 TP=8 shard with Zipf routing, and Qwen3-30B-A3B with MXFP8
weights).  No dataset is involved: activations and weights are random with
the stated distributions, routing is random with the stated law.

Two generators:

* ``make_host_inputs`` -- numpy PCG64, bit-reproducible on any machine; used
  for golden fixtures and CPU-checked parity cases.
* ``make_device_inputs`` -- torch on the GPU (same distributions), used where
  hundreds of MB of weights are needed quickly (bench, full-size tests).

The reference's own inputs (benchmark/bench.py:86-98 of
Religious-J/warp_decode) are unscaled ``randn`` weights with
``rand()``-normalised scales; the configuration distributions below replace
them.  Routing laws:

* ``uniform`` -- each token picks ``topk`` distinct experts uniformly
  (the reference bench's ``rand(B, E).topk(topk)`` law, bench.py:94-95),
* ``zipf``    -- distinct experts drawn without replacement with
  P(rank r) ~ r^-1.1 over a fixed random rank->expert map,
* ``randint`` -- independent uniform draws, duplicates allowed (the law of
  the reference's correctness tests, tests/test_gate_up_correctness.py:52).
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np


@dataclasses.dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    inter: int          # per-GPU intermediate size
    E: int
    topk: int
    routing: str = "uniform"
    weights: str = "bf16"  # or "mxfp8"
    batches: tuple = (1,)
    inter_full: Optional[int] = None  # unsplit intermediate size (tensor-parallel configs)


CONFIGS = {
    # BASELINE configs[0] / [1]: Qwen3-235B-A22B MoE FFN, TP=8 shard.
    "qwen3_235b_tp8": MoEConfig("qwen3_235b_tp8", 4096, 192, 128, 8, "uniform", "bf16",
                                (1, 2, 4, 8, 16, 32, 64), 1536),
    # full width, inter split across 1/2/4/8 GPUs.
    "qwen3_235b_full": MoEConfig("qwen3_235b_full", 4096, 1536, 128, 8, "uniform", "bf16",
                                 (1, 4, 16, 64), 1536),
    # DeepSeek-V3 shard, Zipf(1.1) routing.
    "dsv3_tp8": MoEConfig("dsv3_tp8", 7168, 256, 256, 8, "zipf", "bf16", (1, 8, 32), 2048),
    # Qwen3-30B-A3B with MXFP8 weights.
    "qwen3_30b_mxfp8": MoEConfig("qwen3_30b_mxfp8", 2048, 768, 128, 8, "uniform", "mxfp8",
                                 (1, 2, 4, 8, 16), 768),
}

ZIPF_S = 1.1


# ---------------------------------------------------------------------------
# numpy (host) generation
# ---------------------------------------------------------------------------
def _bf16_bits(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def zipf_rank_map(E: int, seed: int) -> np.ndarray:
    """Fixed random map rank -> expert id for Zipf routing."""
    return np.random.default_rng(np.random.PCG64(seed ^ 0x5A17)).permutation(E)


def host_routing(rng: np.random.Generator, B: int, E: int, topk: int, law: str,
                 seed: int = 0) -> np.ndarray:
    if law == "uniform":
        keys = rng.random((B, E))
        ids = np.argsort(keys, axis=1, kind="stable")[:, :topk]
    elif law == "zipf":
        # Sampling without replacement proportional to r^-s (Gumbel top-k).
        logp = -ZIPF_S * np.log(np.arange(1, E + 1, dtype=np.float64))
        g = -np.log(-np.log(rng.random((B, E)) + 1e-300) + 1e-300)
        ranks = np.argsort(-(logp[None, :] + g), axis=1, kind="stable")[:, :topk]
        ids = zipf_rank_map(E, seed)[ranks]
    elif law == "randint":
        ids = rng.integers(0, E, size=(B, topk))
    else:
        raise ValueError(law)
    return np.ascontiguousarray(ids, dtype=np.int32)


def host_scales(rng: np.random.Generator, B: int, topk: int) -> np.ndarray:
    logits = rng.standard_normal((B, topk))
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    return (p / p.sum(axis=1, keepdims=True)).astype(np.float32)


def host_expert_weights(e: int, hidden: int, inter: int, seed: int, w_std: float,
                        wd_std: float):
    """Weights of one expert from its own PCG64 stream (seed, e): gate_up, down."""
    rng = np.random.default_rng(np.random.SeedSequence([seed, int(e), 7]))
    w_gu = _bf16_bits(rng.standard_normal((2 * inter, hidden), dtype=np.float32) * w_std)
    w_dn = _bf16_bits(rng.standard_normal((hidden, inter), dtype=np.float32) * wd_std)
    return w_gu, w_dn


def make_host_inputs(B: int, hidden: int, inter: int, E: int, topk: int, seed: int = 0,
                     routing: str = "uniform", x_std: float = 1.0,
                     w_std: Optional[float] = None, wd_std: Optional[float] = None,
                     full: bool = False) -> dict:
    """x, routing and scales from one PCG64 stream; weights per touched expert.

    Only experts that appear in topk_ids get weights (each from its own
    stream, so the values do not depend on which other experts are touched).
    ``full=False`` returns the weights as {expert: array}; ``full=True``
    returns dense [E, ...] arrays with zeros for untouched experts (never read
    by any implementation of the path).
    """
    rng = np.random.default_rng(np.random.PCG64(seed))
    w_std = hidden ** -0.5 if w_std is None else w_std
    wd_std = inter ** -0.5 if wd_std is None else wd_std
    x = _bf16_bits(rng.standard_normal((B, hidden), dtype=np.float32) * x_std)
    ids = host_routing(rng, B, E, topk, routing, seed)
    scale = host_scales(rng, B, topk)
    touched = [int(e) for e in np.unique(ids)]
    if full:
        w_gu = np.zeros((E, 2 * inter, hidden), dtype=np.uint16)
        w_dn = np.zeros((E, hidden, inter), dtype=np.uint16)
    else:
        w_gu, w_dn = {}, {}
    for e in touched:
        w_gu[e], w_dn[e] = host_expert_weights(e, hidden, inter, seed, w_std, wd_std)
    return dict(x=x, w_gate_up=w_gu, w_down=w_dn, topk_ids=ids, topk_scale=scale,
                touched=touched)


def input_digest(inp: dict) -> str:
    """SHA-256 over x, routing, scales and the touched experts' weights."""
    import hashlib

    h = hashlib.sha256()
    for k in ("x", "topk_ids", "topk_scale"):
        h.update(np.ascontiguousarray(inp[k]).tobytes())
    for e in inp["touched"]:
        h.update(np.ascontiguousarray(inp["w_gate_up"][e]).tobytes())
        h.update(np.ascontiguousarray(inp["w_down"][e]).tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# torch (device) generation
# ---------------------------------------------------------------------------
def device_routing(B: int, E: int, topk: int, law: str, gen, device, seed: int = 0):
    import torch

    if law == "uniform":
        ids = torch.rand(B, E, generator=gen, device=device).topk(topk, dim=1).indices
    elif law == "zipf":
        logp = -ZIPF_S * torch.log(torch.arange(1, E + 1, device=device, dtype=torch.float64))
        u = torch.rand(B, E, generator=gen, device=device, dtype=torch.float64)
        g = -torch.log(-torch.log(u + 1e-300) + 1e-300)
        ranks = (logp[None, :] + g).topk(topk, dim=1).indices
        rank_map = torch.as_tensor(zipf_rank_map(E, seed), device=device, dtype=torch.int64)
        ids = rank_map[ranks]
    elif law == "randint":
        ids = torch.randint(0, E, (B, topk), generator=gen, device=device)
    else:
        raise ValueError(law)
    return ids.to(torch.int32).contiguous()


def device_scales(B: int, topk: int, gen, device):
    import torch

    logits = torch.randn(B, topk, generator=gen, device=device)
    return torch.softmax(logits, dim=1).float().contiguous()


def make_device_weights(hidden: int, inter: int, E: int, seed: int, device="cuda"):
    """Weights ~ N(0, fan_in^-1/2) generated on the device (bf16)."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w_gu = torch.empty(E, 2 * inter, hidden, device=device, dtype=torch.bfloat16)
    w_dn = torch.empty(E, hidden, inter, device=device, dtype=torch.bfloat16)
    # chunked to bound the fp32 temporary
    for e in range(E):
        w_gu[e] = (torch.randn(2 * inter, hidden, generator=gen, device=device) * hidden ** -0.5).bfloat16()
        w_dn[e] = (torch.randn(hidden, inter, generator=gen, device=device) * inter ** -0.5).bfloat16()
    return w_gu, w_dn


def make_device_activations(B: int, hidden: int, E: int, topk: int, routing: str, seed: int,
                            device="cuda"):
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn(B, hidden, generator=gen, device=device).bfloat16()
    ids = device_routing(B, E, topk, routing, gen, device, seed)
    scale = device_scales(B, topk, gen, device)
    return x, ids, scale


# ---------------------------------------------------------------------------
# Roofline byte model (algorithmic bytes: each touched weight byte once)
# ---------------------------------------------------------------------------
def unique_experts(topk_ids) -> int:
    return int(np.unique(np.asarray(topk_ids).reshape(-1)).size)


def algorithmic_bytes(U: int, B: int, hidden: int, inter: int, topk: int,
                      weights: str = "bf16") -> dict:
    """Bytes a perfect implementation moves per call, split by kernel.

    U experts touched; weights read once each.  gate_up: U*2*I*H weights
    (+ ue8m0 scales for MXFP8), x, ids, h write.  down: U*H*I weights
    (+ scales), h read, ids + scales, y write.
    """
    wb = 1 if weights == "mxfp8" else 2
    sb = 1 if weights == "mxfp8" else 0
    gu_w = U * 2 * inter * hidden * wb + U * 2 * inter * (hidden // 32) * sb
    dn_w = U * hidden * inter * wb + U * hidden * (inter // 32) * sb
    gate_up_b = gu_w + B * hidden * 2 + B * topk * 4 + B * topk * inter * 2
    down_b = dn_w + B * topk * inter * 2 + B * topk * 8 + B * hidden * 2
    return {"gate_up": gate_up_b, "down": down_b, "e2e": gate_up_b + down_b,
            "gate_up_weights": gu_w, "down_weights": dn_w}


def flops(B: int, hidden: int, inter: int, topk: int) -> int:
    return 2 * B * topk * 3 * inter * hidden
