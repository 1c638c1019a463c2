"""The MXFP8 quantise-once loader against the oracle's OCP MX restatement (CPU)."""
import numpy as np
import torch

from oracle import moe_ref as O
from warp_decode_b200.mxfp8 import dequantize_mxfp8, quantize_mxfp8


def test_quantizer_bit_exact_vs_oracle():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((3, 64, 512)) * 0.04).astype(np.float32)
    w[0, 0, :32] = 0.0            # all-zero block -> scale byte 0
    w[1, 2, 5] = 1e-30            # tiny element (flushes to zero at its block's scale)
    w[2, 7, 64:96] *= 1e4         # large block
    wt = torch.from_numpy(w).bfloat16()
    q, s = quantize_mxfp8(wt)
    qo, so = O.mx_quantize(wt.float().numpy())
    assert np.array_equal(q.numpy(), qo)
    assert np.array_equal(s.numpy(), so)
    assert np.array_equal(dequantize_mxfp8(q, s).numpy(), O.mx_dequantize(qo, so))


def test_shapes():
    q, s = quantize_mxfp8(torch.randn(4, 6, 64))
    assert q.dtype == torch.uint8 and s.dtype == torch.uint8
    assert q.shape == (4, 6, 64) and s.shape == (4, 6, 2)
