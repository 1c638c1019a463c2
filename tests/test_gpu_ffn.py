"""Single-launch MoE FFN (wd_moe_ffn_3d_batched) vs the oracle (B200).

The entry point computes moe_down(moe_gate_up(x)) — the two calls the
reference's callers make back to back (benchmark/bench.py:205,254-255 of
Religious-J/warp_decode) — in one cooperative launch: the SIMT kernel for up
to 64 routed slots, the tensor-core kernel (moe_ffn_tc_kernel, the bodies of
the two tcgen05 kernels with one grid barrier between) up to 64 tokens.  Checked through the C ABI: y within rtol = atol = 1e-2 of the
FP32-accumulated oracle, h bit-identical to the SIMT gate_up kernel, the split
(two-kernel) path within the same tolerance, invalid expert ids, subgroups
above the 8-member cap, FP32 output, caller-owned grid-barrier words, and
CUDA-graph replay (the barrier words are reused by every replay).
"""
import numpy as np
import pytest
import torch

from conftest import bf16_close
from oracle import moe_ref as O
from warp_decode_b200 import capi
from warp_decode_b200 import workloads as W

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def wd():
    from warp_decode_b200 import warp_decode

    yield warp_decode
    capi.set_ffn_path(capi.FFN_AUTO)
    warp_decode.set_gate_up_path(capi.GATE_UP_AUTO)


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def check(ours, ref, what):
    ok, dmax = bf16_close(ours, ref, RTOL, ATOL)
    assert ok, f"{what}: max |diff| {dmax:.3e} exceeds atol {ATOL} + rtol {RTOL}*|ref|"


def run_ffn(path, x, wgu, wdn, ids, scale, sync=None, out_fp32=False):
    """y, h and the status word of one wd_moe_ffn_3d_batched call on `path`."""
    B, K = ids.shape
    E, two_i, H = wgu.shape
    I = two_i // 2
    h = torch.empty(B * K, I, dtype=torch.bfloat16, device=x.device)
    y = torch.empty(B, H, dtype=torch.float32 if out_fp32 else torch.bfloat16, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    capi.set_ffn_path(path)
    try:
        capi.check(capi.ffn(x.data_ptr(), wgu.data_ptr(), wdn.data_ptr(), ids.data_ptr(),
                            scale.data_ptr(), h.data_ptr(),
                            None if sync is None else sync.data_ptr(), y.data_ptr(),
                            1 if out_fp32 else 0, B, E, K, H, I, status.data_ptr(),
                            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
    finally:
        capi.set_ffn_path(capi.FFN_AUTO)
    return y, h, int(status.item())


def oracle(x, wgu, wdn, ids, scale):
    ids_h = ids.cpu().numpy()
    E = wgu.shape[0]
    bad = (ids_h < 0) | (ids_h >= E)
    ids_v = np.where(bad, 0, ids_h)
    sc = np.where(bad, 0.0, scale.cpu().numpy()).astype(np.float32)
    touched = lambda w: {int(e): host_bits(w[int(e)]) for e in np.unique(ids_v)}
    h = O.gate_up(host_bits(x), touched(wgu), ids_v)
    h[bad.reshape(-1)] = 0
    return h, O.down(h, touched(wdn), ids_v, sc)


_w = {}


def weights(H, I, E, seed):
    key = (H, I, E, seed)
    if key not in _w:
        _w.clear()
        _w[key] = W.make_device_weights(H, I, E, seed)
    return _w[key]


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16])
def test_qwen3_tp8(wd, B):
    c = W.CONFIGS["qwen3_235b_tp8"]
    wgu, wdn = weights(c.hidden, c.inter, c.E, 41)
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 8100 + B)
    y, h, st = run_ffn(capi.FFN_FUSED, x, wgu, wdn, ids, scale)
    assert st == 0
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    check(host_bits(h), h_ref, f"h B={B}")
    check(host_bits(y), y_ref, f"y B={B}")
    # h is the SIMT gate_up kernel's result, bit for bit (same chunking).
    wd.set_gate_up_path(capi.GATE_UP_SIMT)
    try:
        h_simt = wd.moe_gate_up_3d_batched(x, wgu, ids)
    finally:
        wd.set_gate_up_path(capi.GATE_UP_AUTO)
    if B * c.topk <= 64:
        assert np.array_equal(host_bits(h), host_bits(h_simt))
    y_split, _, st = run_ffn(capi.FFN_SPLIT, x, wgu, wdn, ids, scale)
    assert st == 0
    check(host_bits(y_split), y_ref, f"split y B={B}")
    # torch entry point = the same kernel
    capi.set_ffn_path(capi.FFN_FUSED)
    try:
        y_t = wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
        torch.cuda.synchronize()
    finally:
        capi.set_ffn_path(capi.FFN_AUTO)
    assert np.array_equal(host_bits(y_t), host_bits(y))
    # automatic choice: SIMT single launch up to 32 routed slots, the two
    # kernels up to 64, the tensor-core single launch above
    y_auto, _, st = run_ffn(capi.FFN_AUTO, x, wgu, wdn, ids, scale)
    assert st == 0
    if B * c.topk <= 32:
        assert np.array_equal(host_bits(y_auto), host_bits(y))
    elif B * c.topk <= 64:
        assert np.array_equal(host_bits(y_auto), host_bits(y_split))
    else:
        y_tc, _, st = run_ffn(capi.FFN_TC, x, wgu, wdn, ids, scale)
        assert st == 0
        assert np.array_equal(host_bits(y_auto), host_bits(y_tc))


# (B, hidden, inter, E, topk, routing): ragged rows per CTA, small and large
# inter, top-1, Zipf repeats, experts shared by more than 8 slots.
SHAPES = [
    (3, 2048, 768, 64, 8, "uniform"),
    (1, 7168, 256, 256, 8, "zipf"),
    (4, 7168, 256, 256, 8, "zipf"),
    (2, 1000, 40, 16, 6, "uniform"),
    (1, 4096, 192, 128, 1, "uniform"),
    (8, 4096, 192, 4, 4, "uniform"),
    (16, 512, 64, 2, 2, "uniform"),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:5])) + s[5])
def test_shapes(wd, shape):
    B, H, I, E, K, law = shape
    wgu, wdn = weights(H, I, E, 43)
    x, ids, scale = W.make_device_activations(B, H, E, K, law, 8300 + B)
    y, h, st = run_ffn(capi.FFN_FUSED, x, wgu, wdn, ids, scale)
    assert st == 0
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    check(host_bits(h), h_ref, f"h {shape}")
    check(host_bits(y), y_ref, f"y {shape}")


def test_invalid_ids(wd):
    B, H, I, E, K = 4, 4096, 192, 128, 8
    wgu, wdn = weights(H, I, E, 41)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 8400)
    ids[0, 1] = -1
    ids[2, 7] = E + 5
    y, h, st = run_ffn(capi.FFN_FUSED, x, wgu, wdn, ids, scale)
    assert st & capi.WD_STATUS_BAD_EXPERT_ID
    assert not st & capi.WD_STATUS_WAIT_TIMEOUT
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    hb = host_bits(h)
    assert np.all(hb[0 * K + 1] == 0) and np.all(hb[2 * K + 7] == 0)
    check(hb, h_ref, "h next to invalid ids")
    check(host_bits(y), y_ref, "y with invalid ids")


def test_fp32_out_and_own_sync_words(wd):
    B, H, I, E, K = 2, 4096, 192, 128, 8
    wgu, wdn = weights(H, I, E, 41)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 8500)
    sync = torch.zeros(1, dtype=torch.int64, device="cuda")
    y32, _, st = run_ffn(capi.FFN_FUSED, x, wgu, wdn, ids, scale, sync=sync, out_fp32=True)
    assert st == 0
    U = 4096  # GRID_BAR_UNITS: what one single-launch call adds, whatever its grid
    assert sync.item() == U, "barrier counter: GRID_BAR_UNITS per launch"
    y16, _, st = run_ffn(capi.FFN_FUSED, x, wgu, wdn, ids, scale, sync=sync)
    assert st == 0 and sync.item() == 2 * U
    assert np.array_equal(host_bits(y32.to(torch.bfloat16)), host_bits(y16))
    _, y_ref = oracle(x, wgu, wdn, ids, scale)
    check(host_bits(y16), y_ref, "fp32 output")


def test_graph_replay_and_determinism(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    wgu, wdn = weights(c.hidden, c.inter, c.E, 41)
    B = 8
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 8600)
    capi.set_ffn_path(capi.FFN_FUSED)
    try:
        eager = [host_bits(wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)) for _ in range(3)]
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y_g = wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
        outs = []
        for _ in range(5):
            g.replay()
            torch.cuda.synchronize()
            outs.append(host_bits(y_g).copy())
        del g
    finally:
        capi.set_ffn_path(capi.FFN_AUTO)
    assert wd.status(True, torch.cuda.current_device()) == 0
    for o in eager[1:] + outs:
        assert np.array_equal(o, eager[0])


def test_launch_count(wd):
    """wd_launch_count: one launch per call on the single-launch path, two when
    the FFN runs as gate_up + down, and none for a graph replay."""
    c = W.CONFIGS["qwen3_235b_tp8"]
    wgu, wdn = weights(c.hidden, c.inter, c.E, 41)
    x, ids, scale = W.make_device_activations(2, c.hidden, c.E, c.topk, c.routing, 8700)
    for path, n in ((capi.FFN_FUSED, 1), (capi.FFN_SPLIT, 2)):
        capi.set_ffn_path(path)
        try:
            n0 = wd.launch_count()
            wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
            assert wd.launch_count() - n0 == n
        finally:
            capi.set_ffn_path(capi.FFN_AUTO)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    n0 = wd.launch_count()
    with torch.cuda.graph(g, stream=s):
        wd.moe_ffn_3d_batched(x, wgu, wdn, ids, scale)
    recorded = wd.launch_count() - n0
    g.replay()
    torch.cuda.synchronize()
    assert recorded == 1 and wd.launch_count() - n0 == 1
    del g
    assert wd.status(True, torch.cuda.current_device()) == 0


# ---- tensor-core single launch (FFN_TC: moe_ffn_tc_kernel) ------------------
@pytest.mark.parametrize("B", [1, 4, 8, 16, 33, 64])
def test_tc_single_launch_qwen3(wd, B):
    """y and h against the oracle, one launch per call, y within the
    tolerance of the two-kernel path."""
    c = W.CONFIGS["qwen3_235b_tp8"]
    wgu, wdn = weights(c.hidden, c.inter, c.E, 41)
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 8800 + B)
    n0 = wd.launch_count()
    y, h, st = run_ffn(capi.FFN_TC, x, wgu, wdn, ids, scale)
    assert st == 0
    assert wd.launch_count() - n0 == 1, "one launch for the whole FFN"
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    check(host_bits(h), h_ref, f"tc h B={B}")
    check(host_bits(y), y_ref, f"tc y B={B}")
    y_split, _, st = run_ffn(capi.FFN_SPLIT, x, wgu, wdn, ids, scale)
    assert st == 0
    check(host_bits(y), host_bits(y_split), f"tc vs split B={B}")


# (B, hidden, inter, E, topk, routing): several down stages per item (inter
# 768), 56 row tiles (hidden 7168), Zipf repeats with experts shared by more
# than 16 slots (down items cut in runs of 16), top-1, ragged inter.
TC_SHAPES = [
    (3, 2048, 768, 64, 8, "uniform"),
    (16, 2048, 768, 128, 8, "uniform"),
    (4, 7168, 256, 256, 8, "zipf"),
    (32, 7168, 256, 256, 8, "zipf"),
    (48, 4096, 192, 16, 8, "uniform"),
    (20, 4096, 192, 128, 1, "uniform"),
    (9, 1024, 72, 32, 4, "uniform"),
]


@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "x".join(map(str, s[:5])) + s[5])
def test_tc_single_launch_shapes(wd, shape):
    B, H, I, E, K, law = shape
    wgu, wdn = weights(H, I, E, 47)
    x, ids, scale = W.make_device_activations(B, H, E, K, law, 8900 + B)
    n0 = wd.launch_count()
    y, h, st = run_ffn(capi.FFN_TC, x, wgu, wdn, ids, scale)
    assert st == 0
    assert wd.launch_count() - n0 == 1
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    check(host_bits(h), h_ref, f"tc h {shape}")
    check(host_bits(y), y_ref, f"tc y {shape}")


def test_tc_single_launch_invalid_ids(wd):
    B, H, I, E, K = 16, 4096, 192, 128, 8
    wgu, wdn = weights(H, I, E, 41)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 9000)
    ids[0, 1] = -1
    ids[9, 7] = E + 5
    y, h, st = run_ffn(capi.FFN_TC, x, wgu, wdn, ids, scale)
    assert st & capi.WD_STATUS_BAD_EXPERT_ID
    assert not st & capi.WD_STATUS_WAIT_TIMEOUT
    h_ref, y_ref = oracle(x, wgu, wdn, ids, scale)
    hb = host_bits(h)
    assert np.all(hb[0 * K + 1] == 0) and np.all(hb[9 * K + 7] == 0)
    check(hb, h_ref, "tc h next to invalid ids")
    check(host_bits(y), y_ref, "tc y with invalid ids")


def test_tc_and_simt_single_launch_share_the_barrier(wd):
    """The two single-launch kernels (grids of different sizes) take turns on
    one grid-barrier counter, caller-owned and library-owned, eagerly and in
    a CUDA graph; every result stays the same."""
    c = W.CONFIGS["qwen3_235b_tp8"]
    wgu, wdn = weights(c.hidden, c.inter, c.E, 41)
    xa, ia, sa = W.make_device_activations(2, c.hidden, c.E, c.topk, c.routing, 9100)
    xb, ib, sb = W.make_device_activations(16, c.hidden, c.E, c.topk, c.routing, 9116)
    sync = torch.zeros(1, dtype=torch.int64, device="cuda")
    ya0, _, st = run_ffn(capi.FFN_FUSED, xa, wgu, wdn, ia, sa, sync=sync)
    assert st == 0
    yb0, _, st = run_ffn(capi.FFN_TC, xb, wgu, wdn, ib, sb, sync=sync)
    assert st == 0
    assert sync.item() == 2 * 4096
    for s_ in (sync, None):
        for _ in range(2):
            ya, _, st = run_ffn(capi.FFN_FUSED, xa, wgu, wdn, ia, sa, sync=s_)
            assert st == 0 and np.array_equal(host_bits(ya), host_bits(ya0))
            yb, _, st = run_ffn(capi.FFN_TC, xb, wgu, wdn, ib, sb, sync=s_)
            assert st == 0 and np.array_equal(host_bits(yb), host_bits(yb0))
    capi.set_ffn_path(capi.FFN_AUTO)  # B=2: SIMT single launch, B=16: tensor-core
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        wd.moe_ffn_3d_batched(xa, wgu, wdn, ia, sa)
        wd.moe_ffn_3d_batched(xb, wgu, wdn, ib, sb)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ga = wd.moe_ffn_3d_batched(xa, wgu, wdn, ia, sa)
        gb = wd.moe_ffn_3d_batched(xb, wgu, wdn, ib, sb)
    for _ in range(4):
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(host_bits(ga), host_bits(ya0))
        assert np.array_equal(host_bits(gb), host_bits(yb0))
    del g
    assert wd.status(True, torch.cuda.current_device()) == 0
