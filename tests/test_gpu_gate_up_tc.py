"""tcgen05 tensor-core gate_up vs the oracle and vs the SIMT kernel (B200).

Both kernels implement moe_gate_up_3d_batched (csrc/moe_gate_up_3d_batched.cu
of Religious-J/warp_decode); the path is forced with wd_set_gate_up_path so
each one is checked at every shape, including the batch sizes where the
automatic choice would pick the other.  Tolerance: bf16 outputs within
rtol = atol = 1e-2 of the FP32-accumulated oracle.
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
    warp_decode.set_gate_up_path(capi.GATE_UP_AUTO)


def dev_bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def check(ours, ref, what):
    ok, dmax = bf16_close(ours, ref, RTOL, ATOL)
    assert ok, f"{what}: max |diff| {dmax:.3e} exceeds atol {ATOL} + rtol {RTOL}*|ref|"


def run_path(wd, path, x, w, ids):
    wd.set_gate_up_path(path)
    try:
        h = wd.moe_gate_up_3d_batched(x, w, ids)
        torch.cuda.synchronize()
        assert wd.status(True, torch.cuda.current_device()) == 0
    finally:
        wd.set_gate_up_path(capi.GATE_UP_AUTO)
    return h


_w = {}


def qwen_weights():
    if "q" not in _w:
        c = W.CONFIGS["qwen3_235b_tp8"]
        _w["q"] = W.make_device_weights(c.hidden, c.inter, c.E, 21)[0]
    return _w["q"]


@pytest.mark.parametrize("B", [1, 2, 4, 16, 64])
def test_qwen3_tp8_both_paths(wd, B):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_weights()
    x, ids, _ = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 5000 + B)
    h_tc = run_path(wd, capi.GATE_UP_TC, x, w, ids)
    h_simt = run_path(wd, capi.GATE_UP_SIMT, x, w, ids)
    ids_h = ids.cpu().numpy()
    touched = {int(e): host_bits(w[int(e)]) for e in np.unique(ids_h)}
    ref = O.gate_up(host_bits(x), touched, ids_h)
    check(host_bits(h_tc), ref, "tcgen05 gate_up")
    check(host_bits(h_simt), ref, "SIMT gate_up")


@pytest.mark.parametrize("B,E,K,H,I,routing", [
    (3, 5, 3, 264, 48, "randint"),      # hidden % 64 != 0 (zero-filled K tail), partial tile
    (2, 1, 4, 128, 16, "randint"),      # one expert, inter far below one 64-neuron tile
    (3, 5, 3, 264, 40, "randint"),      # inter % 16 != 0
    (64, 2, 8, 256, 32, "randint"),     # ~256 slots per expert: groups split at 64 members
    (5, 6, 6, 128, 80, "randint"),      # duplicate ids inside a token
    (100, 64, 8, 512, 64, "uniform"),   # B*topk > 512: two launches
    (4, 2048, 8, 256, 64, "uniform"),   # E > 1024: tensor-core path does not apply (SIMT)
    (8, 256, 8, 7168, 256, "zipf"),     # DeepSeek-V3 TP=8 shard shape, skewed routing
])
def test_shapes_tc(wd, B, E, K, H, I, routing):
    inp = W.make_host_inputs(B, H, I, E, K, seed=B * 11 + E, routing=routing, full=True)
    x, w = dev_bf16(inp["x"]), dev_bf16(inp["w_gate_up"])
    ids = torch.from_numpy(inp["topk_ids"]).cuda()
    h = run_path(wd, capi.GATE_UP_TC, x, w, ids)
    ref = O.gate_up(inp["x"], inp["w_gate_up"], inp["topk_ids"])
    check(host_bits(h), ref, "tcgen05 gate_up")


def test_invalid_ids_tc(wd):
    B, E, K, H, I = 6, 16, 4, 256, 64
    inp = W.make_host_inputs(B, H, I, E, K, seed=77, routing="uniform", full=True)
    ids_h = inp["topk_ids"].copy()
    ids_h[1, 2] = E          # out of range
    ids_h[4, 0] = -3         # negative
    x, w = dev_bf16(inp["x"]), dev_bf16(inp["w_gate_up"])
    ids = torch.from_numpy(ids_h).cuda()
    wd.set_gate_up_path(capi.GATE_UP_TC)
    try:
        wd.status(True, torch.cuda.current_device())
        h = wd.moe_gate_up_3d_batched(x, w, ids)
        torch.cuda.synchronize()
        st = wd.status(True, torch.cuda.current_device())
    finally:
        wd.set_gate_up_path(capi.GATE_UP_AUTO)
    assert st & 0x1, "BAD_EXPERT_ID must be raised"
    assert not st & 0x2, "no wait may time out"
    hb = host_bits(h)
    for (b, s) in [(1, 2), (4, 0)]:
        assert np.all(hb[b * K + s] == 0), "slot with an invalid id must be zeros"
    ok_ids = ids_h.copy()
    ok_ids[1, 2] = 0
    ok_ids[4, 0] = 0
    ref = O.gate_up(inp["x"], inp["w_gate_up"], ok_ids)
    mask = np.ones(B * K, bool)
    mask[[1 * K + 2, 4 * K + 0]] = False
    check(hb[mask], ref[mask], "valid slots next to invalid ones")


def test_graph_replay_tc(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_weights()
    B = 16
    x, ids, _ = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 6001)
    wd.set_gate_up_path(capi.GATE_UP_TC)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for _ in range(2):
                wd.moe_gate_up_3d_batched(x, w, ids)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            h = wd.moe_gate_up_3d_batched(x, w, ids)
        x2, ids2, _ = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 6002)
        x.copy_(x2)
        ids.copy_(ids2)
        g.replay()
        torch.cuda.synchronize()
        assert wd.status(True, torch.cuda.current_device()) == 0
    finally:
        wd.set_gate_up_path(capi.GATE_UP_AUTO)
    ids_h = ids.cpu().numpy()
    touched = {int(e): host_bits(w[int(e)]) for e in np.unique(ids_h)}
    check(host_bits(h), O.gate_up(host_bits(x), touched, ids_h), "graph replay, new routing")


def test_deterministic_tc(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w = qwen_weights()
    x, ids, _ = W.make_device_activations(32, c.hidden, c.E, c.topk, c.routing, 6100)
    a = run_path(wd, capi.GATE_UP_TC, x, w, ids)
    b = run_path(wd, capi.GATE_UP_TC, x, w, ids)
    assert torch.equal(a, b)


# ---------------------------------------------------------------------------
# MXFP8 weights on the tensor cores (E4M3 decoded to bf16 on chip)
# ---------------------------------------------------------------------------
E4M3_FINITE = np.array([b for b in range(256) if b & 0x7F != 0x7F], dtype=np.uint8)


def run_mx(wd, path, x, q, s, ids):
    wd.set_gate_up_path(path)
    try:
        wd.status(True, torch.cuda.current_device())
        h = wd.moe_gate_up_3d_batched_mxfp8(x, q, s, ids)
        torch.cuda.synchronize()
        st = wd.status(True, torch.cuda.current_device())
    finally:
        wd.set_gate_up_path(capi.GATE_UP_AUTO)
    return h, st


def mx_oracle(x, q, s, ids_h):
    """The oracle on the dequantised weights of every valid touched expert."""
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    E = q.shape[0]
    touched = {int(e): dequantize_mxfp8(q[int(e)], s[int(e)]).cpu().numpy()
               for e in np.unique(ids_h) if 0 <= e < E}
    return O.gate_up(host_bits(x), touched, ids_h)


def mx_weights(E, I, H, seed):
    from warp_decode_b200.mxfp8 import quantize_mxfp8

    key = ("mx", E, I, H, seed)
    if key not in _w:
        for k in [k for k in _w if k != "q"]:
            del _w[k]
        torch.cuda.empty_cache()
        w = W.make_device_weights(H, I, E, seed)[0]
        _w[key] = quantize_mxfp8(w)
        del w
    return _w[key]


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16])
def test_mxfp8_qwen3_30b_both_paths(wd, B):
    c = W.CONFIGS["qwen3_30b_mxfp8"]
    q, s = mx_weights(c.E, c.inter, c.hidden, 31)
    x, ids, _ = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 7000 + B)
    h_tc, st_tc = run_mx(wd, capi.GATE_UP_TC, x, q, s, ids)
    h_simt, st_simt = run_mx(wd, capi.GATE_UP_SIMT, x, q, s, ids)
    assert st_tc == 0 and st_simt == 0
    ref = mx_oracle(x, q, s, ids.cpu().numpy())
    check(host_bits(h_tc), ref, "tcgen05 MXFP8 gate_up vs oracle on dequantised weights")
    check(host_bits(h_simt), ref, "SIMT MXFP8 gate_up vs oracle on dequantised weights")


@pytest.mark.parametrize("B,E,K,H,I,routing", [
    (3, 5, 3, 512, 40, "randint"),      # partial neuron tile, duplicates inside a token
    (1, 4, 1, 1024, 64, "uniform"),     # one item: K split over a cluster
    (32, 128, 8, 4096, 192, "uniform"), # two launches of 16 tokens
    (8, 256, 8, 7168, 256, "zipf"),     # DeepSeek-V3 shard shape, skewed routing
])
def test_mxfp8_shapes_tc(wd, B, E, K, H, I, routing):
    q, s = mx_weights(E, I, H, 7 + E)
    x, ids, _ = W.make_device_activations(B, H, E, K, routing, 7100 + B)
    h, st = run_mx(wd, capi.GATE_UP_TC, x, q, s, ids)
    assert st == 0
    check(host_bits(h), mx_oracle(x, q, s, ids.cpu().numpy()), "tcgen05 MXFP8 gate_up")


def test_mxfp8_tc_decodes_every_byte_like_simt(wd):
    """One-hot x: h[b, n] = silu(Wg[n, b]) * Wu[n, b] is a single product, so
    both kernels are exact up to the same final rounding and must agree bit
    for bit, over every finite E4M3 byte and block scales on both sides of
    the one-multiply limit (scale byte 134)."""
    rng = np.random.default_rng(23)
    B, I, H = 64, 128, 512
    q = rng.choice(E4M3_FINITE, size=(1, 2 * I, H)).astype(np.uint8)
    k = np.arange(E4M3_FINITE.size)
    q[0, k // B, k % B] = rng.permutation(E4M3_FINITE)
    s = rng.choice(np.array([100, 127, 134, 135, 150], dtype=np.uint8), size=(1, 2 * I, H // 32))
    q, s = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    x = torch.zeros(B, H, dtype=torch.bfloat16, device="cuda")
    x[torch.arange(B), torch.arange(B)] = 1.0
    ids = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    h_tc, st_tc = run_mx(wd, capi.GATE_UP_TC, x, q, s, ids)
    h_simt, st_simt = run_mx(wd, capi.GATE_UP_SIMT, x, q, s, ids)
    assert st_tc == 0 and st_simt == 0
    assert torch.equal(h_tc, h_simt)
    check(host_bits(h_tc), mx_oracle(x, q, s, ids.cpu().numpy()), "one-hot x")


def test_mxfp8_tc_nan_and_invalid_ids(wd):
    """A NaN byte (gate row) and a NaN scale byte 255 (up row) make exactly
    those neurons NaN for the slots of that expert, as on the SIMT kernel;
    out-of-range expert ids give zero rows and BAD_EXPERT_ID."""
    B, E, K, H, I = 4, 8, 2, 1024, 64
    q, s = mx_weights(E, I, H, 99)
    q, s = q.clone(), s.clone()
    x, ids, _ = W.make_device_activations(B, H, E, K, "uniform", 7300)
    ids[2, 1] = E
    ids[3, 0] = -1
    e0 = int(ids[0, 0])
    q[e0, 5, 700] = 0x7F   # gate row of neuron 5
    s[e0, I + 9, 3] = 255  # up row of neuron 9
    h_tc, st_tc = run_mx(wd, capi.GATE_UP_TC, x, q, s, ids)
    h_simt, st_simt = run_mx(wd, capi.GATE_UP_SIMT, x, q, s, ids)
    assert st_tc & 0x1 and st_simt & 0x1 and not st_tc & 0x2
    nan_tc, nan_simt = torch.isnan(h_tc.float()), torch.isnan(h_simt.float())
    assert torch.equal(nan_tc, nan_simt) and nan_tc.any()
    ids_h = ids.cpu().numpy()
    slots = [b * K + j for b in range(B) for j in range(K) if ids_h[b, j] == e0]
    assert nan_tc[slots][:, [5, 9]].all()
    hb = host_bits(h_tc)
    assert np.all(hb[2 * K + 1] == 0) and np.all(hb[3 * K + 0] == 0)
    ok = ~nan_tc.cpu().numpy()
    valid = np.ones(B * K, bool)
    valid[[2 * K + 1, 3 * K + 0]] = False
    ref = mx_oracle(x, q, s, np.where((ids_h >= 0) & (ids_h < E), ids_h, 0))
    check(hb[valid][ok[valid]], ref[valid][ok[valid]], "finite outputs next to NaN ones")
