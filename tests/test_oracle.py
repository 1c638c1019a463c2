"""The oracle against the reference itself (CPU only).

The golden fixtures hold outputs of the reference's own PyTorch functions
(``reference_gate_up``, ``reference_down`` and the FP32 formula of
tests/test_benchmark_reference.py:36-43 of Religious-J/warp_decode) on
seeded inputs; ``oracle.moe_ref`` must reproduce them.  The reference's bmm
accumulates in FP32 in its own order and the oracle evaluates each projection
exactly before rounding, so a few outputs may differ in the last bf16 bit.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_close, golden_array, golden_cases, golden_inputs
from oracle import moe_ref as O

CASES = golden_cases()


def _agree(ours, ref):
    exact = float((ours == ref).mean())
    ok, dmax = bf16_close(ours, ref, rtol=2 ** -7, atol=1e-3)
    return exact, ok, dmax


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_oracle_matches_reference(case, mode):
    inp = golden_inputs(case)
    n = case["name"]
    h = O.gate_up(inp["x"], inp["w_gate_up"], inp["topk_ids"], mode=mode)
    exact, ok, dmax = _agree(h, golden_array(f"{n}/h_{mode}"))
    assert ok and exact > 0.995, (exact, dmax)
    # down is checked on the reference's own h so the two stages pin separately
    y = O.down(golden_array(f"{n}/h_{mode}"), inp["w_down"], inp["topk_ids"], inp["topk_scale"],
               mode=mode)
    exact, ok, dmax = _agree(y, golden_array(f"{n}/y_{mode}"))
    assert ok and exact > 0.995, (exact, dmax)


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    f = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 100000),
                        np.array([0.0, -0.0, 1.0, 65504.0, 3.4e38, 1e-40], dtype=np.float32)])
    ours = O.f32_to_bf16(f)
    ref = torch.from_numpy(f).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)
    assert np.array_equal(O.bf16_to_f32(ours), torch.from_numpy(ours.view(np.int16)).view(torch.bfloat16).float().numpy())


def test_e4m3_matches_torch_float8():
    # every finite E4M3 value decodes like torch's float8_e4m3fn
    codes = np.arange(256, dtype=np.uint8)
    finite = (codes & 0x7F) != 0x7F
    ours = O.e4m3_to_f32(codes)[finite]
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()[finite]
    assert np.array_equal(ours, ref)
    # rounding of arbitrary values inside the finite range equals torch's cast
    rng = np.random.default_rng(1)
    v = np.clip(rng.standard_normal(200000) * 10.0 ** rng.uniform(-4, 2.6, 200000), -448, 448)
    v = np.concatenate([v, O.e4m3_to_f32(codes)[finite].astype(np.float64)]).astype(np.float32)
    ours = O.f32_to_e4m3(v)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)


def test_mx_quantize_properties():
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((64, 256)) * 0.03).astype(np.float32)
    w[3, :32] = 0.0  # an all-zero block
    q, s = O.mx_quantize(w)
    assert q.shape == w.shape and s.shape == (64, 8)
    deq = O.mx_dequantize(q, s)
    blocks = w.reshape(64, 8, 32)
    amax = np.abs(blocks).max(-1)
    # shared exponent = floor(log2(amax)) - 8 (OCP MX v1.0, emax(E4M3) = 8)
    nz = amax > 0
    assert np.array_equal(s[nz].astype(int) - 127, (np.floor(np.log2(amax[nz])) - 8).astype(int))
    assert np.all(deq[3, :32] == 0.0)
    # E4M3 keeps 3 mantissa bits: error <= half a step (2^-4 relative for
    # normals, 2^-10 * X for subnormals); scaled values above 448 saturate
    # (the shared exponent maps a block maximum into [256, 512)).
    err = np.abs(deq - w).astype(np.float64)
    X = np.repeat(np.exp2(s.astype(np.float64) - 127), 32, axis=1)
    sat = np.abs(w) / X > O.E4M3_MAX
    bound = np.maximum(np.abs(w) * 2.0 ** -4, X * 2.0 ** -10)
    assert np.all(err[~sat] <= bound[~sat] * 1.0001)
    np.testing.assert_allclose(err[sat], np.abs(w[sat]) - O.E4M3_MAX * X[sat], rtol=1e-6)
    assert np.all(np.abs(deq[sat]) == O.E4M3_MAX * X[sat])


def test_oracle_invariants():
    # permuting the top-k slots of a token (ids and scales together) keeps y
    rng = np.random.default_rng(3)
    from warp_decode_b200.workloads import make_host_inputs

    inp = make_host_inputs(4, 256, 64, 16, 4, seed=5)
    h = O.gate_up(inp["x"], inp["w_gate_up"], inp["topk_ids"])
    y = O.down(h, inp["w_down"], inp["topk_ids"], inp["topk_scale"], return_f32=True)
    perm = rng.permutation(4)
    ids_p = inp["topk_ids"][:, perm]
    h_p = h.reshape(4, 4, 64)[:, perm].reshape(16, 64)
    y_p = O.down(h_p, inp["w_down"], ids_p, inp["topk_scale"][:, perm], return_f32=True)
    np.testing.assert_allclose(y_p, y, rtol=1e-6, atol=1e-6)
