"""tcgen05 tensor-core down vs the oracle and vs the SIMT kernel (B200).

Both kernels implement moe_down_3d_batched (csrc/moe_down_3d_batched.cu of
Religious-J/warp_decode); the path is forced with wd_set_down_path.  The
down kernel is fed a fixed bf16 h so it is judged on its own.  Tolerance:
bf16 outputs within rtol = atol = 1e-2 of the FP32-accumulated oracle.
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
    warp_decode.set_down_path(capi.PATH_AUTO)


def dev_bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def check(ours, ref, what):
    ok, dmax = bf16_close(ours, ref, RTOL, ATOL)
    assert ok, f"{what}: max |diff| {dmax:.3e} exceeds atol {ATOL} + rtol {RTOL}*|ref|"


def run_down(wd, path, h, w, ids, scale, B, partial=False):
    wd.set_down_path(path)
    try:
        fn = wd.moe_down_3d_batched_partial if partial else wd.moe_down_3d_batched
        y = fn(h, w, ids, scale, B)
        torch.cuda.synchronize()
        st = wd.status(True, torch.cuda.current_device())
    finally:
        wd.set_down_path(capi.PATH_AUTO)
    return y, st


def random_h(n, inter, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(n, inter, generator=g) * 0.5).to(torch.bfloat16).cuda()


_w = {}


def qwen_down():
    if "q" not in _w:
        c = W.CONFIGS["qwen3_235b_tp8"]
        _w["q"] = W.make_device_weights(c.hidden, c.inter, c.E, 31)[1]
    return _w["q"]


@pytest.mark.parametrize("B", [1, 2, 4, 16, 64])
def test_qwen3_tp8_both_paths(wd, B):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_down()
    _, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 7000 + B)
    h = random_h(B * c.topk, c.inter, 7100 + B)
    y_tc, st_tc = run_down(wd, capi.PATH_TC, h, w, ids, scale, B)
    y_simt, st_simt = run_down(wd, capi.PATH_SIMT, h, w, ids, scale, B)
    assert st_tc == 0 and st_simt == 0
    ids_h = ids.cpu().numpy()
    touched = {int(e): host_bits(w[int(e)]) for e in np.unique(ids_h)}
    ref = O.down(host_bits(h), touched, ids_h, scale.cpu().numpy())
    check(host_bits(y_tc), ref, "tcgen05 down")
    check(host_bits(y_simt), ref, "SIMT down")


@pytest.mark.parametrize("B,E,K,H,I,routing", [
    (3, 5, 3, 264, 40, "randint"),      # inter % 64 != 0 (zero K tail), hidden % 128 != 0
    (2, 1, 4, 128, 8, "randint"),       # one expert, inter = 8
    (64, 2, 8, 256, 32, "randint"),     # ~256 slots per expert: items of 16 members
    (5, 6, 6, 128, 64, "randint"),      # repeated ids inside a token (fixed add order)
    (100, 64, 8, 512, 64, "uniform"),   # B*topk > 512: two launches
    (4, 2048, 8, 256, 64, "uniform"),   # E > 1024: SIMT path
    (2, 16, 4, 512, 1544, "uniform"),   # 25 K chunks (last partial) in h slices of 4
    (2, 16, 4, 512, 2056, "uniform"),   # inter > 2048: SIMT path
    (16, 64, 8, 1024, 1536, "uniform"), # Qwen3-235B full width (TP1): 6 stages per item
    (6, 16, 4, 512, 1000, "uniform"),   # 16 K chunks over 4 weight stages, last chunk partial
    (9, 32, 8, 1024, 512, "randint"),   # 2 weight stages per item, repeated ids
    (8, 256, 8, 7168, 256, "zipf"),     # DeepSeek-V3 TP=8 shard: 56 tiles, clusters of 2
    (16, 128, 8, 2048, 768, "uniform"), # Qwen3-30B shape, bf16: 3 weight stages per item
])
def test_shapes_tc(wd, B, E, K, H, I, routing):
    inp = W.make_host_inputs(B, H, I, E, K, seed=B * 13 + E, routing=routing, full=True)
    w = dev_bf16(inp["w_down"])
    ids = torch.from_numpy(inp["topk_ids"]).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    h = random_h(B * K, I, B * 17 + I)
    y, st = run_down(wd, capi.PATH_TC, h, w, ids, scale, B)
    assert st == 0
    ref = O.down(host_bits(h), inp["w_down"], inp["topk_ids"], inp["topk_scale"])
    check(host_bits(y), ref, "tcgen05 down")


def test_invalid_ids_tc(wd):
    B, E, K, H, I = 6, 16, 4, 256, 64
    inp = W.make_host_inputs(B, H, I, E, K, seed=78, routing="uniform", full=True)
    ids_h = inp["topk_ids"].copy()
    ids_h[1, 2] = E
    ids_h[4, 0] = -3
    w = dev_bf16(inp["w_down"])
    ids = torch.from_numpy(ids_h).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    h = random_h(B * K, I, 79)
    wd.status(True, torch.cuda.current_device())
    y, st = run_down(wd, capi.PATH_TC, h, w, ids, scale, B)
    assert st & 0x1 and not st & 0x2
    # invalid slots contribute nothing: same as a zero scale on a valid expert
    ok_ids = ids_h.copy()
    ok_ids[1, 2] = 0
    ok_ids[4, 0] = 0
    sc = inp["topk_scale"].copy()
    sc[1, 2] = 0.0
    sc[4, 0] = 0.0
    ref = O.down(host_bits(h), inp["w_down"], ok_ids, sc)
    check(host_bits(y), ref, "invalid slots skipped")


def test_fp32_partial_tc(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_down()
    B = 8
    _, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 7200)
    h = random_h(B * c.topk, c.inter, 7201)
    y32, st = run_down(wd, capi.PATH_TC, h, w, ids, scale, B, partial=True)
    assert st == 0 and y32.dtype == torch.float32
    y16, _ = run_down(wd, capi.PATH_TC, h, w, ids, scale, B)
    assert torch.equal(y32.to(torch.bfloat16), y16)
    ids_h = ids.cpu().numpy()
    touched = {int(e): host_bits(w[int(e)]) for e in np.unique(ids_h)}
    ref = O.down(host_bits(h), touched, ids_h, scale.cpu().numpy(), return_f32=True)
    np.testing.assert_allclose(y32.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


def test_graph_replay_and_determinism_tc(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_down()
    B = 32
    _, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 7300)
    h = random_h(B * c.topk, c.inter, 7301)
    wd.set_down_path(capi.PATH_TC)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for _ in range(2):
                wd.moe_down_3d_batched(h, w, ids, scale, B)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y = wd.moe_down_3d_batched(h, w, ids, scale, B)
        _, ids2, scale2 = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 7302)
        ids.copy_(ids2)
        scale.copy_(scale2)
        g.replay()
        torch.cuda.synchronize()
        first = y.clone()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(first, y)
        assert wd.status(True, torch.cuda.current_device()) == 0
    finally:
        wd.set_down_path(capi.PATH_AUTO)
    ids_h = ids.cpu().numpy()
    touched = {int(e): host_bits(w[int(e)]) for e in np.unique(ids_h)}
    check(host_bits(y), O.down(host_bits(h), touched, ids_h, scale.cpu().numpy()),
          "graph replay, new routing")


# ---------------------------------------------------------------------------
# MXFP8 weights on the tensor cores (E4M3 decoded to bf16 on chip)
# ---------------------------------------------------------------------------
E4M3_FINITE = np.array([b for b in range(256) if b & 0x7F != 0x7F], dtype=np.uint8)


def run_down_mx(wd, path, h, q, s, ids, scale, B):
    wd.set_down_path(path)
    try:
        wd.status(True, torch.cuda.current_device())
        y = wd.moe_down_3d_batched_mxfp8(h, q, s, ids, scale, B)
        torch.cuda.synchronize()
        st = wd.status(True, torch.cuda.current_device())
    finally:
        wd.set_down_path(capi.PATH_AUTO)
    return y, st


def mx_down_oracle(h, q, s, ids_h, scale_h):
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    E = q.shape[0]
    touched = {int(e): dequantize_mxfp8(q[int(e)], s[int(e)]).cpu().numpy()
               for e in np.unique(ids_h) if 0 <= e < E}
    return O.down(host_bits(h), touched, ids_h, scale_h)


def mx_down_weights(E, H, I, seed):
    from warp_decode_b200.mxfp8 import quantize_mxfp8

    key = ("mxd", E, H, I, seed)
    if key not in _w:
        for k in [k for k in _w if isinstance(k, tuple) and k[0] == "mxd"]:
            del _w[k]
        torch.cuda.empty_cache()
        w = W.make_device_weights(H, I, E, seed)[1]
        _w[key] = quantize_mxfp8(w)
        del w
    return _w[key]


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16, 32])
def test_mxfp8_qwen3_30b_both_paths(wd, B):
    c = W.CONFIGS["qwen3_30b_mxfp8"]
    q, s = mx_down_weights(c.E, c.hidden, c.inter, 33)
    _, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 8000 + B)
    h = random_h(B * c.topk, c.inter, 8100 + B)
    y_tc, st_tc = run_down_mx(wd, capi.PATH_TC, h, q, s, ids, scale, B)
    y_simt, st_simt = run_down_mx(wd, capi.PATH_SIMT, h, q, s, ids, scale, B)
    assert st_tc == 0 and st_simt == 0
    ref = mx_down_oracle(h, q, s, ids.cpu().numpy(), scale.cpu().numpy())
    check(host_bits(y_tc), ref, "tcgen05 MXFP8 down vs oracle on dequantised weights")
    check(host_bits(y_simt), ref, "SIMT MXFP8 down vs oracle on dequantised weights")


@pytest.mark.parametrize("B,E,K,H,I,routing", [
    (3, 5, 3, 256, 128, "randint"),     # one 128-K box per item, duplicates inside a token
    (8, 256, 8, 7168, 256, "zipf"),     # DeepSeek-V3 shard shape, skewed routing
    (4, 16, 8, 1024, 2048, "uniform"),  # inter at the tensor-core limit: 4 weight stages per item
])
def test_mxfp8_shapes_tc(wd, B, E, K, H, I, routing):
    q, s = mx_down_weights(E, H, I, 9 + E)
    _, ids, scale = W.make_device_activations(B, H, E, K, routing, 8200 + B)
    h = random_h(B * K, I, 8300 + B)
    y, st = run_down_mx(wd, capi.PATH_TC, h, q, s, ids, scale, B)
    assert st == 0
    check(host_bits(y), mx_down_oracle(h, q, s, ids.cpu().numpy(), scale.cpu().numpy()),
          "tcgen05 MXFP8 down")


def test_mxfp8_tc_reads_back_every_byte_exactly(wd):
    """One-hot h rows: y[b, n] = W[n, b] exactly (one product per output),
    over every finite E4M3 byte and block scales on both sides of the
    one-multiply limit (scale byte 134), through 128 / 16 launches."""
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    rng = np.random.default_rng(29)
    H, I = 256, 128
    B = I
    q = rng.choice(E4M3_FINITE, size=(1, H, I)).astype(np.uint8)
    q.reshape(-1)[: E4M3_FINITE.size] = rng.permutation(E4M3_FINITE)
    s = rng.choice(np.array([100, 127, 134, 135, 150], dtype=np.uint8), size=(1, H, I // 32))
    q, s = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    h = torch.eye(B, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    scale = torch.ones(B, 1, dtype=torch.float32, device="cuda")
    y, st = run_down_mx(wd, capi.PATH_TC, h, q, s, ids, scale, B)
    assert st == 0
    want = dequantize_mxfp8(q, s)[0].t()  # [B, H]
    assert torch.equal(want.to(torch.bfloat16).float(), want), "test weights exact in bf16"
    bad = (y.float() != want).nonzero()
    assert bad.numel() == 0, f"{bad.shape[0]} mismatches, first at {bad[0].tolist()}"


def test_mxfp8_tc_nan_and_invalid_ids(wd):
    """A NaN byte and a NaN scale byte make exactly their output rows NaN for
    the tokens routed to that expert (as on the SIMT kernel); out-of-range
    ids contribute nothing and raise BAD_EXPERT_ID."""
    B, E, K, H, I = 4, 8, 2, 512, 256
    q, s = mx_down_weights(E, H, I, 77)
    q, s = q.clone(), s.clone()
    _, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 8400)
    ids[3, 1] = E
    e0 = int(ids[0, 0])
    q[e0, 7, 100] = 0x7F
    s[e0, 300, 2] = 255
    h = random_h(B * K, I, 8401)
    y_tc, st_tc = run_down_mx(wd, capi.PATH_TC, h, q, s, ids, scale, B)
    y_simt, st_simt = run_down_mx(wd, capi.PATH_SIMT, h, q, s, ids, scale, B)
    assert st_tc & 0x1 and st_simt & 0x1 and not st_tc & 0x2
    nan_tc, nan_simt = torch.isnan(y_tc.float()), torch.isnan(y_simt.float())
    assert torch.equal(nan_tc, nan_simt)
    toks = sorted({b for b in range(B) for j in range(K) if int(ids[b, j]) == e0})
    assert nan_tc[toks][:, [7, 300]].all()
    ids_h = ids.cpu().numpy()
    sc_h = scale.cpu().numpy().copy()
    sc_h[ids_h >= E] = 0.0
    ref = mx_down_oracle(h, q, s, np.where(ids_h < E, ids_h, (e0 + 1) % E), sc_h)
    ok = ~nan_tc.cpu().numpy()
    check(host_bits(y_tc)[ok], ref[ok], "finite outputs next to NaN ones")
