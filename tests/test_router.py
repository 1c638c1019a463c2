"""Router producer (wd_moe_router_topk): top-k experts and routing weights.

No counterpart in the reference (it takes topk_ids / topk_scale as inputs).
CPU: the numpy restatement against torch.topk / torch.softmax, and the C-ABI
argument checks.  GPU: the kernel against the restatement — ids exact,
weights within rtol 1e-6 / atol 1e-7 (FP32 expf against float64) — for bf16
and fp32 logits, with and without renormalisation, ties, NaN and -inf
logits, and the shapes of the benchmark configs.
"""
import numpy as np
import pytest
import torch

from oracle import moe_ref as O
from warp_decode_b200 import capi


def test_oracle_matches_torch():
    g = torch.Generator().manual_seed(3)
    lg = torch.randn(16, 128, generator=g)
    ids, w = O.router_topk(lg.numpy(), 8, True)
    tv, ti = torch.topk(lg, 8, dim=1)
    assert np.array_equal(ids, ti.numpy())
    assert np.allclose(w, torch.softmax(tv.double(), dim=1).numpy(), rtol=1e-6, atol=1e-7)
    ids2, w2 = O.router_topk(lg.numpy(), 8, False)
    assert np.array_equal(ids2, ids)
    full = torch.softmax(lg.double(), dim=1).numpy()
    assert np.allclose(w2, np.take_along_axis(full, ids2, axis=1), rtol=1e-6, atol=1e-7)


def test_oracle_ties_and_nan():
    lg = np.array([[1.0, 3.0, 3.0, np.nan, -np.inf, 3.0]], dtype=np.float32)
    ids, w = O.router_topk(lg, 5, True)
    # NaN ranks as -inf; equal values (3.0 x 3, -inf x 2) in ascending expert order
    assert ids.tolist() == [[1, 2, 5, 0, 3]]
    assert abs(w.sum() - 1.0) < 1e-6 and w[0, 4] == 0.0


def test_router_validates_before_touching_the_device():
    L = capi.lib()
    assert capi.router_topk(16, 1, 16, 16, 4, 8, 9, 1) == capi.WD_ERR_SHAPE   # topk > E
    assert capi.router_topk(16, 1, 16, 16, 4, 2048, 8, 1) == capi.WD_ERR_UNSUPPORTED
    assert capi.router_topk(16, 1, 16, 16, 4, 128, 33, 1) == capi.WD_ERR_UNSUPPORTED
    assert capi.router_topk(None, 1, 16, 16, 4, 128, 8, 1) == capi.WD_ERR_NULL_POINTER
    assert capi.router_topk(18, 1, 16, 16, 4, 128, 8, 1) == capi.WD_ERR_ALIGNMENT
    assert b"misaligned" in L.wd_last_error_message()
    assert capi.router_topk(None, 1, None, None, 0, 128, 8, 1) == capi.WD_OK


CASES = [  # (B, E, topk, dtype, renormalize)
    (1, 128, 8, torch.bfloat16, True),
    (64, 128, 8, torch.bfloat16, True),
    (33, 256, 8, torch.float32, True),
    (17, 128, 8, torch.float32, False),
    (5, 1000, 32, torch.float32, True),
    (9, 40, 1, torch.bfloat16, False),
    (3, 8, 8, torch.float32, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}E{c[1]}k{c[2]}{str(c[3])[6:]}r{int(c[4])}")
def test_router_kernel(case):
    from warp_decode_b200 import warp_decode as wd

    B, E, K, dt, ren = case
    g = torch.Generator().manual_seed(B * 1000 + E + K)
    lg = torch.randn(B, E, generator=g).to(dt)
    if B > 2:  # ties (bf16 makes many more), a NaN and a -inf
        lg[1, 3] = lg[1, 5]
        lg[2, 0] = float("nan")
        lg[2, 1] = float("-inf")
    ids, w = wd.moe_router_topk(lg.cuda(), K, ren)
    torch.cuda.synchronize()
    ids_r, w_r = O.router_topk(lg.float().numpy(), K, ren)
    assert np.array_equal(ids.cpu().numpy(), ids_r)
    assert np.allclose(w.cpu().numpy(), w_r, rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
def test_router_feeds_the_ffn():
    """Router output goes straight into the FFN entry point."""
    from warp_decode_b200 import warp_decode as wd
    from warp_decode_b200 import workloads as W

    H, I, E, K, B = 1024, 64, 32, 4, 4
    wgu, wdn = W.make_device_weights(H, I, E, 61)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16).cuda()
    lg = torch.randn(B, E, generator=g).cuda()
    ids, w = wd.moe_router_topk(lg, K, True)
    y = wd.moe_ffn_3d_batched(x, wgu, wdn, ids, w)
    torch.cuda.synchronize()
    ids_r, w_r = O.router_topk(lg.cpu().numpy(), K, True)
    assert np.array_equal(ids.cpu().numpy(), ids_r)
    bits = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    touched = lambda wt: {int(e): bits(wt[int(e)]) for e in np.unique(ids_r)}
    h = O.gate_up(bits(x), touched(wgu), ids_r)
    y_ref = O.down(h, touched(wdn), ids_r, w_r)
    from conftest import bf16_close
    ok, d = bf16_close(bits(y), y_ref, 1e-2, 1e-2)
    assert ok, d
