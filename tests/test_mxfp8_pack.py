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


def _packed(tmp_path, E=3, H=64, I=32, seed=1):
    g = torch.Generator().manual_seed(seed)
    w_gu = (torch.randn(E, 2 * I, H, generator=g) * H ** -0.5).bfloat16()
    w_dn = (torch.randn(E, H, I, generator=g) * I ** -0.5).bfloat16()
    return tmp_path / "moe.wdmx", w_gu, w_dn


def test_file_round_trip_is_bit_exact(tmp_path):
    from warp_decode_b200.mxfp8 import load_mxfp8, load_or_quantize_moe

    path, w_gu, w_dn = _packed(tmp_path)
    gq, gs, dq, ds = load_or_quantize_moe(str(path), w_gu, w_dn)  # quantises and writes
    assert path.exists()
    t, meta = load_mxfp8(str(path))
    assert meta == {"experts": 3, "hidden": 64, "inter": 32}
    for (a, b), (c, d) in ((t["w_gate_up"], (gq, gs)), (t["w_down"], (dq, ds))):
        assert torch.equal(a, c) and torch.equal(b, d)
    # the second call loads (no weights needed) and matches the oracle's quantiser
    gq2, gs2, dq2, ds2 = load_or_quantize_moe(str(path))
    qo, so = O.mx_quantize(w_gu.float().numpy())
    assert np.array_equal(gq2.numpy(), qo) and np.array_equal(gs2.numpy(), so)
    qo, so = O.mx_quantize(w_dn.float().numpy())
    assert np.array_equal(dq2.numpy(), qo) and np.array_equal(ds2.numpy(), so)


def test_file_rejects_mismatches(tmp_path):
    import struct

    import pytest

    from warp_decode_b200.mxfp8 import load_mxfp8, load_or_quantize_moe

    path, w_gu, w_dn = _packed(tmp_path)
    load_or_quantize_moe(str(path), w_gu, w_dn)
    raw = path.read_bytes()
    bad = tmp_path / "bad.wdmx"

    def rejects(data, match):
        bad.write_bytes(data)
        with pytest.raises(ValueError, match=match):
            load_mxfp8(str(bad))

    rejects(b"XXXX" + raw[4:], "magic")
    rejects(raw[:4] + struct.pack("<I", 2) + raw[8:], "version")
    rejects(raw[:-1000], "size")
    flipped = bytearray(raw)
    flipped[-3] ^= 0x40  # a payload byte of the last scale array
    rejects(bytes(flipped), "checksum")
    hlen = struct.unpack("<I", raw[8:12])[0]
    hdr = raw[12:12 + hlen].replace(b'"block": 32', b'"block": 16')
    rejects(raw[:12] + hdr + raw[12 + hlen:], "block")
    # a file for another layer shape
    with pytest.raises(ValueError, match="shape"):
        load_or_quantize_moe(str(path), w_gu[:, :, :32], w_dn[:, :32, :])
