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
