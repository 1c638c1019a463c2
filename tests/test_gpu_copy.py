"""GPU-driven host <-> device transfers (wd_copy_ranges) and the host-buffer
FFN entry point built on them (moe_ffn_3d_batched_host), on a B200.

Byte-exact copies in both directions and device to device, at sizes around
the 16-byte unit (0, 1, 15, 16, 17, ...) and at unaligned offsets, up to four
ranges in one launch; pageable host memory is refused before any launch; the
host-buffer FFN returns the same bits as moe_ffn_3d_batched on the same
inputs, on every kernel path (B = 1, 8, 16, 64), eagerly and replayed from a
CUDA graph.
"""
import pytest
import torch

from warp_decode_b200 import capi
from warp_decode_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wd():
    from warp_decode_b200 import warp_decode

    return warp_decode


def pinned_bytes(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g).pin_memory()


@pytest.mark.parametrize("n", [1, 15, 16, 17, 255, 4096 + 3, 1 << 20])
@pytest.mark.parametrize("offset", [0, 1, 8])
def test_round_trip_bytes(wd, n, offset):
    src = pinned_bytes(n + offset + 16, n + offset)
    dev = torch.full((n + offset + 16,), 0xAB, dtype=torch.uint8, device="cuda")
    back = torch.zeros(n + offset + 16, dtype=torch.uint8).pin_memory()
    wd.copy_ranges([src[offset:offset + n]], [dev[offset:offset + n]])
    wd.copy_ranges([dev[offset:offset + n]], [back[offset:offset + n]])
    torch.cuda.synchronize()
    assert torch.equal(dev[offset:offset + n].cpu(), src[offset:offset + n])
    assert torch.equal(back[offset:offset + n], src[offset:offset + n])
    # bytes outside the ranges are untouched
    assert torch.all(dev[:offset].cpu() == 0xAB) and torch.all(dev[offset + n:].cpu() == 0xAB)
    assert torch.all(back[:offset] == 0) and torch.all(back[offset + n:] == 0)


def test_four_ranges_one_launch(wd):
    sizes = [8192, 256, 3, 100_000]
    srcs = [pinned_bytes(s, i) for i, s in enumerate(sizes)]
    dsts = [torch.empty(s, dtype=torch.uint8, device="cuda") for s in sizes]
    n0 = wd.launch_count()
    wd.copy_ranges(srcs, dsts)
    assert wd.launch_count() - n0 == 1
    torch.cuda.synchronize()
    for s, d in zip(srcs, dsts):
        assert torch.equal(d.cpu(), s)


def test_device_to_device_and_empty(wd):
    a = torch.arange(1000, dtype=torch.int32, device="cuda")
    b = torch.zeros_like(a)
    wd.copy_ranges([a, a[:0]], [b, b[:0]])
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # only empty ranges: nothing launched
    n0 = wd.launch_count()
    wd.copy_ranges([a[:0]], [b[:0]])
    assert wd.launch_count() == n0


def test_pageable_host_memory_refused(wd):
    pageable = torch.zeros(64, dtype=torch.uint8)
    dev = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="pinned"):
        wd.copy_ranges([pageable], [dev])
    # the C ABI itself refuses pageable memory before launching
    n0 = wd.launch_count()
    rc = capi.copy_ranges([pageable.data_ptr()], [dev.data_ptr()], [64])
    assert rc == capi.WD_ERR_UNSUPPORTED
    assert "pageable" in capi.lib().wd_last_error_message().decode()
    assert wd.launch_count() == n0
    torch.cuda.synchronize()


def test_mismatched_sizes_refused(wd):
    a = pinned_bytes(32, 1)
    b = torch.zeros(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="sizes differ"):
        wd.copy_ranges([a], [b])


@pytest.mark.parametrize("B", [1, 8, 16, 64])
def test_host_ffn_matches_device_ffn(wd, B):
    H, I, E, K = 4096, 192, 128, 8
    w_gu, w_dn = W.make_device_weights(H, I, E, 11)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 100 + B)
    want = wd.moe_ffn_3d_batched(x, w_gu, w_dn, ids, scale)
    xh, idh, sch = x.cpu().pin_memory(), ids.cpu().pin_memory(), scale.cpu().pin_memory()
    got = wd.moe_ffn_3d_batched_host(xh, w_gu, w_dn, idh, sch)
    torch.cuda.synchronize()
    assert got.device.type == "cpu" and got.is_pinned()
    assert torch.equal(got.view(torch.int16), want.cpu().view(torch.int16))
    # caller-owned output, replayed from a CUDA graph
    out = torch.zeros_like(got).pin_memory()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        wd.moe_ffn_3d_batched_host(xh, w_gu, w_dn, idh, sch, out=out)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        wd.moe_ffn_3d_batched_host(xh, w_gu, w_dn, idh, sch, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), want.cpu().view(torch.int16))
    del g


def test_host_ffn_empty_batch(wd):
    H, I, E, K = 256, 64, 8, 2
    w_gu, w_dn = W.make_device_weights(H, I, E, 3)
    x = torch.zeros(0, H, dtype=torch.bfloat16).pin_memory()
    ids = torch.zeros(0, K, dtype=torch.int32).pin_memory()
    scale = torch.zeros(0, K, dtype=torch.float32).pin_memory()
    y = wd.moe_ffn_3d_batched_host(x, w_gu, w_dn, ids, scale)
    assert tuple(y.shape) == (0, H)


def test_host_ffn_rejects_device_inputs(wd):
    H, I, E, K = 256, 64, 8, 2
    w_gu, w_dn = W.make_device_weights(H, I, E, 3)
    x, ids, scale = W.make_device_activations(2, H, E, K, "uniform", 4)
    with pytest.raises(RuntimeError, match="pinned host"):
        wd.moe_ffn_3d_batched_host(x, w_gu, w_dn, ids, scale)
