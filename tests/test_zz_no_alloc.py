"""wd_moe_ffn_3d_batched_noalloc: the single-launch FFN with its scratch (h and
the grid-barrier counter) in a static device array of the library.

Collected last.  On CPU: oversize requests are rejected before any device
call.  On a B200: two calls in a row through the C ABI give the same bits as
the existing entry point (wd_moe_ffn_3d_batched, caller-owned h and counter)
on the same inputs, at a single-launch size and at a two-kernel size.
"""
import numpy as np
import pytest
import torch

from warp_decode_b200 import capi
from warp_decode_b200 import workloads as W


def test_oversize_is_rejected_without_a_device():
    L = capi.lib()
    # 64 slots x 1032 inter x 2 bytes > 131072
    rc = capi.ffn_noalloc(16, 16, 16, 16, 16, 16, 0, 8, 128, 8, 4096, 1032)
    assert rc == capi.WD_ERR_UNSUPPORTED
    assert b"scratch" in L.wd_last_error_message()
    assert capi.ffn_noalloc(None, None, None, None, None, None, 0, 0, 128, 8, 4096, 192) == capi.WD_OK


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("B", [2, 16])
def test_matches_the_existing_entry_point_twice(B):
    c = W.CONFIGS["qwen3_235b_tp8"]
    H, I, E, K = c.hidden, c.inter, c.E, c.topk
    wgu, wdn = W.make_device_weights(H, I, E, 51)
    x, ids, scale = W.make_device_activations(B, H, E, K, c.routing, 9100 + B)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    h = torch.empty(B * K, I, dtype=torch.bfloat16, device="cuda")
    sync = torch.zeros(1, dtype=torch.int64, device="cuda")
    y_ref = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
    capi.check(capi.ffn(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(), ids.data_ptr(),
                        scale.data_ptr(), h.data_ptr(), sync.data_ptr(), y_ref.data_ptr(), 0, B, E,
                        K, H, I, status.data_ptr(), stream))
    outs = []
    for _ in range(2):
        y = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
        capi.check(capi.ffn_noalloc(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(), ids.data_ptr(),
                                    scale.data_ptr(), y.data_ptr(), 0, B, E, K, H, I,
                                    status.data_ptr(), stream))
        outs.append(y)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for y in outs:
        assert np.array_equal(_bits(y), _bits(y_ref))


@pytest.mark.gpu
def test_scratch_boundary_each_path():
    """h of exactly the scratch size (64 slots x 1024 inter x 2 bytes = 131072)
    on every kernel choice, bit for bit against the existing entry point; one
    token more is refused, and the next in-range call still matches."""
    B, H, I, E, K = 8, 4096, 1024, 16, 8
    assert B * K * I * 2 == 131072
    wgu, wdn = W.make_device_weights(H, I, E, 53)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 9300)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    h = torch.empty(B * K, I, dtype=torch.bfloat16, device="cuda")
    try:
        for path in (capi.FFN_FUSED, capi.FFN_SPLIT, capi.FFN_TC, capi.FFN_AUTO):
            capi.set_ffn_path(path)
            y_ref = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
            capi.check(capi.ffn(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(), ids.data_ptr(),
                                scale.data_ptr(), h.data_ptr(), None, y_ref.data_ptr(), 0, B, E,
                                K, H, I, status.data_ptr(), stream))
            y = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
            capi.check(capi.ffn_noalloc(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(),
                                        ids.data_ptr(), scale.data_ptr(), y.data_ptr(), 0, B, E,
                                        K, H, I, status.data_ptr(), stream))
            torch.cuda.synchronize()
            assert int(status.item()) == 0, f"path {path}"
            assert np.array_equal(_bits(y), _bits(y_ref)), f"path {path}"
            # one more routed slot's worth of h does not fit: refused, nothing launched
            y2 = torch.empty(B + 1, H, dtype=torch.bfloat16, device="cuda")
            x2, ids2, sc2 = W.make_device_activations(B + 1, H, E, K, "uniform", 9301)
            assert capi.ffn_noalloc(x2.data_ptr(), wgu.data_ptr(), wdn.data_ptr(),
                                    ids2.data_ptr(), sc2.data_ptr(), y2.data_ptr(), 0, B + 1, E,
                                    K, H, I, status.data_ptr(), stream) == capi.WD_ERR_UNSUPPORTED
            y3 = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
            capi.check(capi.ffn_noalloc(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(),
                                        ids.data_ptr(), scale.data_ptr(), y3.data_ptr(), 0, B, E,
                                        K, H, I, status.data_ptr(), stream))
            torch.cuda.synchronize()
            assert np.array_equal(_bits(y3), _bits(y_ref)), f"path {path} after a refusal"
    finally:
        capi.set_ffn_path(capi.FFN_AUTO)
