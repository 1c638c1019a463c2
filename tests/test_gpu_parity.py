"""CUDA path vs the oracle and the reference's golden outputs (B200).

Tolerances: bf16 outputs within rtol = atol = 1e-2 of the FP32-accumulated
reference (tests/test_benchmark_reference.py:36-43 of Religious-J/warp_decode);
against the reference's bf16-bmm functions the reference's own test tolerance,
rtol = atol = 5e-2 (tests/test_gate_up_correctness.py:69).  MXFP8: the same
1e-2 against the FP32 oracle run on the dequantised weights (the weights are
exactly representable after dequantisation; only accumulation order differs).
"""
import numpy as np
import pytest
import torch

from conftest import bf16_close, golden_array, golden_cases, golden_inputs
from oracle import moe_ref as O
from warp_decode_b200 import capi
from warp_decode_b200 import workloads as W

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
REF_TOL = 5e-2


@pytest.fixture(scope="module")
def wd():
    from warp_decode_b200 import warp_decode

    return warp_decode


def dev_bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_bf16_close(ours, ref, rtol=RTOL, atol=ATOL, what=""):
    ok, dmax = bf16_close(ours, ref, rtol, atol)
    assert ok, f"{what}: max |diff| {dmax:.3e} exceeds atol {atol} + rtol {rtol}*|ref|"


# ---------------------------------------------------------------------------
# golden fixtures (outputs of the reference's own functions)
# ---------------------------------------------------------------------------
CASES = golden_cases()


@pytest.mark.parametrize("api", ["torch", "capi"])
@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden(wd, case, api):
    inp = golden_inputs(case, full=True)
    n, B = case["name"], case["B"]
    x, w_gu, w_dn = dev_bf16(inp["x"]), dev_bf16(inp["w_gate_up"]), dev_bf16(inp["w_down"])
    ids = torch.from_numpy(inp["topk_ids"]).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    if api == "torch":
        h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
        y_on_ref_h = wd.moe_down_3d_batched(dev_bf16(golden_array(f"{n}/h_fp32")), w_dn, ids, scale, B)
        y = wd.moe_down_3d_batched(h, w_dn, ids, scale, B)
    else:
        h = capi.torch_gate_up(x, w_gu, ids)
        y_on_ref_h = capi.torch_down(dev_bf16(golden_array(f"{n}/h_fp32")), w_dn, ids, scale)
        y = capi.torch_down(h, w_dn, ids, scale)
    torch.cuda.synchronize()
    h, y, y_on_ref_h = host_bits(h), host_bits(y), host_bits(y_on_ref_h)
    assert_bf16_close(h, golden_array(f"{n}/h_fp32"), what="gate_up vs FP32 reference")
    assert_bf16_close(h, golden_array(f"{n}/h_bf16"), REF_TOL, REF_TOL, "gate_up vs reference_gate_up")
    assert_bf16_close(y_on_ref_h, golden_array(f"{n}/y_fp32"), what="down vs FP32 reference")
    assert_bf16_close(y, golden_array(f"{n}/y_fp32"), what="e2e vs FP32 reference")
    assert_bf16_close(y, golden_array(f"{n}/y_bf16"), REF_TOL, REF_TOL, "e2e vs reference_down")


# ---------------------------------------------------------------------------
# benchmark configurations at full size (device-generated weights)
# ---------------------------------------------------------------------------
_weights = {}


def cfg_weights(name, hidden, inter, E, seed):
    key = (name, hidden, inter, E, seed)
    if key not in _weights:
        _weights.clear()
        torch.cuda.empty_cache()
        _weights[key] = W.make_device_weights(hidden, inter, E, seed)
    return _weights[key]


def touched_host(w, ids):
    return {int(e): host_bits(w[int(e)]) for e in torch.unique(ids).tolist()}


def run_and_check(wd, x, w_gu, w_dn, ids, scale):
    B = x.shape[0]
    h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
    y = wd.moe_down_3d_batched(h, w_dn, ids, scale, B)
    torch.cuda.synchronize()
    assert wd.status(True, torch.cuda.current_device()) == 0
    ids_h = ids.cpu().numpy()
    h_ref = O.gate_up(host_bits(x), touched_host(w_gu, ids), ids_h)
    assert_bf16_close(host_bits(h), h_ref, what="gate_up")
    # down is checked on our own h so the two kernels are judged separately
    y_ref = O.down(host_bits(h), touched_host(w_dn, ids), ids_h, scale.cpu().numpy())
    assert_bf16_close(host_bits(y), y_ref, what="down")


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16, 32, 64])
def test_config_qwen3_235b_tp8(wd, B):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w_gu, w_dn = cfg_weights(c.name, c.hidden, c.inter, c.E, 11)
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 1000 + B)
    run_and_check(wd, x, w_gu, w_dn, ids, scale)


@pytest.mark.parametrize("B", [1, 8, 32])
def test_config_dsv3_zipf(wd, B):
    c = W.CONFIGS["dsv3_tp8"]
    w_gu, w_dn = cfg_weights(c.name, c.hidden, c.inter, c.E, 12)
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 2000 + B)
    run_and_check(wd, x, w_gu, w_dn, ids, scale)


@pytest.mark.parametrize("tp,B", [(1, 1), (1, 16), (2, 4), (4, 64)])
def test_config_qwen3_235b_full_shards(wd, tp, B):
    c = W.CONFIGS["qwen3_235b_full"]
    inter = c.inter_full // tp
    w_gu, w_dn = cfg_weights(f"{c.name}/tp{tp}", c.hidden, inter, c.E, 13)
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 3000 + B)
    run_and_check(wd, x, w_gu, w_dn, ids, scale)


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16])
def test_config_qwen3_30b_mxfp8(wd, B):
    from warp_decode_b200.mxfp8 import dequantize_mxfp8, quantize_mxfp8

    c = W.CONFIGS["qwen3_30b_mxfp8"]
    key = ("mx", c.name)
    if key not in _weights:
        _weights.clear()
        torch.cuda.empty_cache()
        w_gu, w_dn = W.make_device_weights(c.hidden, c.inter, c.E, 14)
        _weights[key] = quantize_mxfp8(w_gu) + quantize_mxfp8(w_dn)
    gq, gs, dq, ds = _weights[key]
    x, ids, scale = W.make_device_activations(B, c.hidden, c.E, c.topk, c.routing, 4000 + B)
    h = wd.moe_gate_up_3d_batched_mxfp8(x, gq, gs, ids)
    y = wd.moe_down_3d_batched_mxfp8(h, dq, ds, ids, scale, B)
    torch.cuda.synchronize()
    ids_h = ids.cpu().numpy()
    gu_f = {e: dequantize_mxfp8(gq[e], gs[e]).cpu().numpy() for e in torch.unique(ids).tolist()}
    dn_f = {e: dequantize_mxfp8(dq[e], ds[e]).cpu().numpy() for e in torch.unique(ids).tolist()}
    h_ref = O.gate_up(host_bits(x), gu_f, ids_h)
    assert_bf16_close(host_bits(h), h_ref, what="mxfp8 gate_up vs oracle on dequantised weights")
    y_ref = O.down(host_bits(h), dn_f, ids_h, scale.cpu().numpy())
    assert_bf16_close(host_bits(y), y_ref, what="mxfp8 down vs oracle on dequantised weights")
    # the C ABI entry points give the same bits
    h2 = torch.empty_like(h)
    capi.check(capi.gate_up_mxfp8(x.data_ptr(), gq.data_ptr(), gs.data_ptr(), ids.data_ptr(),
                                  h2.data_ptr(), B, c.E, c.topk, c.hidden, c.inter, None,
                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(h, h2)


E4M3_FINITE = np.array([b for b in range(256) if b & 0x7F != 0x7F], dtype=np.uint8)


def mx_every_byte(rows, cols, seed, scales=(110, 127, 140)):
    """q [1, rows, cols] holding every finite E4M3 encoding (subnormals and
    +-0 included) at least once, block scales drawn from `scales` (dequantised
    values stay normal in bf16, so they are exact there)."""
    rng = np.random.default_rng(seed)
    q = rng.choice(E4M3_FINITE, size=(1, rows, cols)).astype(np.uint8)
    q.reshape(-1)[: E4M3_FINITE.size] = rng.permutation(E4M3_FINITE)
    s = rng.choice(np.array(scales, dtype=np.uint8), size=(1, rows, cols // 32))
    return torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()


@pytest.mark.parametrize("B", [64, 96])
def test_mxfp8_every_e4m3_byte_decodes_exactly(wd, B):
    """down with one-hot h reads the weights back: y[b, n] = W[n, b] exactly,
    for every finite E4M3 byte (the in-register decode is exact), through the
    small (B*topk <= 64) and large routing paths."""
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    H = 256
    q, s = mx_every_byte(H, B, 91 + B)
    h = torch.eye(B, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    scale = torch.ones(B, 1, dtype=torch.float32, device="cuda")
    y = wd.moe_down_3d_batched_mxfp8(h, q, s, ids, scale, B)
    torch.cuda.synchronize()
    want = dequantize_mxfp8(q, s)[0].t()  # [B, H]
    assert torch.equal(want.to(torch.bfloat16).float(), want), "test weights exact in bf16"
    bad = (y.float() != want).nonzero()
    assert bad.numel() == 0, f"{bad.shape[0]} mismatches, first at {bad[0].tolist()}: " \
        f"q byte 0x{int(q[0, bad[0, 1], bad[0, 0]]):02x}"


def test_mxfp8_nan_encoding_propagates(wd):
    """An E4M3 NaN byte (S.1111.111) makes its row's outputs NaN, as the
    dequantised oracle does (NaN * 0 = NaN); every other row stays exact."""
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    B, H = 32, 128
    q, s = mx_every_byte(H, B, 5)
    q[0, 3, 17] = 0x7F
    q[0, 40, 0] = 0xFF
    h = torch.eye(B, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    scale = torch.ones(B, 1, dtype=torch.float32, device="cuda")
    y = wd.moe_down_3d_batched_mxfp8(h, q, s, ids, scale, B).float()
    torch.cuda.synchronize()
    want = dequantize_mxfp8(q, s)[0].t()
    nan_rows = [3, 40]
    assert torch.isnan(y[:, nan_rows]).all()
    keep = [n for n in range(H) if n not in nan_rows]
    assert torch.equal(y[:, keep], want[:, keep])


def test_mxfp8_gate_up_every_e4m3_byte(wd):
    """gate_up with one-hot x: gate and up of token b are single weights, so h
    = silu(W_g[n, b]) * W_u[n, b] over every finite E4M3 byte."""
    from warp_decode_b200.mxfp8 import dequantize_mxfp8

    B, I = 64, 128
    q, s = mx_every_byte(2 * I, B, 17)
    x = torch.eye(B, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    h = wd.moe_gate_up_3d_batched_mxfp8(x, q, s, ids)
    torch.cuda.synchronize()
    w = {0: dequantize_mxfp8(q[0], s[0]).cpu().numpy()}
    h_ref = O.gate_up(host_bits(x), w, ids.cpu().numpy())
    assert_bf16_close(host_bits(h), h_ref, what="mxfp8 gate_up, one-hot x")


# ---------------------------------------------------------------------------
# shapes and edge cases
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("B,E,K,H,I,routing", [
    (1, 4, 2, 256, 8, "randint"),        # smallest reference shape
    (3, 5, 3, 264, 40, "randint"),       # hidden % 256 != 0, inter % 64 != 0 (reference rejects)
    (2, 4, 1, 64, 8, "uniform"),         # topk = 1
    (5, 6, 6, 128, 16, "randint"),       # many duplicates
    (2, 1, 4, 128, 8, "randint"),        # one expert: every slot identical
    (100, 64, 8, 512, 64, "uniform"),    # B*topk = 800 > 512: split into two launches
    (4, 2048, 8, 256, 64, "uniform"),    # E > 1024: per-slot groups
    (2, 16, 8, 7168, 64, "uniform"),     # hidden spans two 8 KB chunks
    (2, 16, 4, 512, 1544, "uniform"),    # large inter, rows per stage < 4...
    (70, 8, 8, 256, 8, "randint"),       # > GROUP_MAX slots per expert
])
def test_shapes_and_edges(wd, B, E, K, H, I, routing):
    inp = W.make_host_inputs(B, H, I, E, K, seed=B * 7 + E, routing=routing, full=True)
    x, w_gu, w_dn = dev_bf16(inp["x"]), dev_bf16(inp["w_gate_up"]), dev_bf16(inp["w_down"])
    ids = torch.from_numpy(inp["topk_ids"]).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
    y = wd.moe_down_3d_batched(h, w_dn, ids, scale, B)
    torch.cuda.synchronize()
    h_ref = O.gate_up(inp["x"], inp["w_gate_up"], inp["topk_ids"])
    assert_bf16_close(host_bits(h), h_ref, what="gate_up")
    y_ref = O.down(host_bits(h), inp["w_down"], inp["topk_ids"], inp["topk_scale"])
    assert_bf16_close(host_bits(y), y_ref, what="down")


def test_empty_batch(wd):
    x = torch.zeros(0, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(4, 16, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(0, 2, dtype=torch.int32, device="cuda")
    h = wd.moe_gate_up_3d_batched(x, w, ids)
    assert h.shape == (0, 8)
    y = wd.moe_down_3d_batched(torch.zeros(0, 64, dtype=torch.bfloat16, device="cuda"),
                               torch.zeros(4, 256, 64, dtype=torch.bfloat16, device="cuda"), ids,
                               torch.zeros(0, 2, device="cuda"), 0)
    assert y.shape == (0, 256)


def test_out_of_range_expert_ids_are_flagged_and_zero(wd):
    B, E, K, H, I = 3, 8, 4, 256, 64
    inp = W.make_host_inputs(B, H, I, E, K, seed=77, full=True)
    ids_np = inp["topk_ids"].copy()
    ids_np[0, 1] = E          # out of range
    ids_np[2, 3] = -5         # negative
    x, w_gu, w_dn = dev_bf16(inp["x"]), dev_bf16(inp["w_gate_up"]), dev_bf16(inp["w_down"])
    ids = torch.from_numpy(ids_np).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    wd.status(True, torch.cuda.current_device())
    h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
    y = wd.moe_down_3d_batched(h, w_dn, ids, scale, B)
    torch.cuda.synchronize()
    st = wd.status(True, torch.cuda.current_device())
    assert st & capi.WD_STATUS_BAD_EXPERT_ID
    hb = host_bits(h)
    assert not hb[0 * K + 1].any() and not hb[2 * K + 3].any()
    # reference semantics for the valid slots; invalid slots contribute nothing
    valid = ids_np.copy()
    valid[0, 1] = valid[0, 0]
    valid[2, 3] = valid[2, 0]
    h_ref = O.gate_up(inp["x"], inp["w_gate_up"], valid)
    h_ref[0 * K + 1] = 0
    h_ref[2 * K + 3] = 0
    assert_bf16_close(hb, h_ref, what="gate_up")
    sc = inp["topk_scale"].copy()
    sc[0, 1] = 0.0
    sc[2, 3] = 0.0
    y_ref = O.down(hb, inp["w_down"], valid, sc)
    assert_bf16_close(host_bits(y), y_ref, what="down")


def test_fp32_partial_output(wd):
    B, E, K, H, I = 4, 16, 8, 512, 128
    inp = W.make_host_inputs(B, H, I, E, K, seed=5, full=True)
    h = dev_bf16(O.gate_up(inp["x"], inp["w_gate_up"], inp["topk_ids"]))
    ids = torch.from_numpy(inp["topk_ids"]).cuda()
    scale = torch.from_numpy(inp["topk_scale"]).cuda()
    y32 = wd.moe_down_3d_batched_partial(h, dev_bf16(inp["w_down"]), ids, scale, B)
    y16 = wd.moe_down_3d_batched(h, dev_bf16(inp["w_down"]), ids, scale, B)
    torch.cuda.synchronize()
    assert y32.dtype == torch.float32
    ref = O.down(host_bits(h), inp["w_down"], inp["topk_ids"], inp["topk_scale"], return_f32=True)
    np.testing.assert_allclose(y32.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)
    assert torch.equal(y32.bfloat16(), y16)


def test_cuda_graph_replay_with_mutated_inputs(wd):
    """The reference's graph-safety pattern (tests/test_benchmark_reference.py:48-66)."""
    c = W.CONFIGS["qwen3_235b_tp8"]
    w_gu, w_dn = cfg_weights(c.name, c.hidden, c.inter, c.E, 11)
    x, ids, scale = W.make_device_activations(8, c.hidden, c.E, c.topk, c.routing, 55)

    def e2e():
        h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
        return wd.moe_down_3d_batched(h, w_dn, ids, scale, 8)

    standard = e2e()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            e2e()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        captured = e2e()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, standard)
    x.mul_(0.5)
    ids.copy_((ids + 1) % c.E)
    updated = e2e()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, updated)
    del graph


def test_deterministic(wd):
    c = W.CONFIGS["qwen3_235b_tp8"]
    w_gu, w_dn = cfg_weights(c.name, c.hidden, c.inter, c.E, 11)
    x, ids, scale = W.make_device_activations(16, c.hidden, c.E, c.topk, "randint", 66)
    outs = []
    for _ in range(3):
        h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
        outs.append(wd.moe_down_3d_batched(h, w_dn, ids, scale, 16))
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
