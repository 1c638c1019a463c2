"""The E4M3 -> bf16 decode of the MXFP8 tensor-core kernels, restated in
numpy and checked against the oracle's OCP MX dequantisation (CPU).

The kernels (`e4m3x16_to_bf16` and `mx_decode_scaled` in
warp_decode_b200/csrc) turn each E4M3 byte into a bf16 bit pattern with one
byte permute (sign replicated into the high byte), a shift by 4 and a mask,
which is the E4M3 value times 2^-120, then multiply in bf16 by 2^(s - 7) for
the block's UE8M0 scale byte s (by 2^127 and then 2^(s - 134) when s > 134,
where 2^(s - 7) is not a bf16 normal); a NaN byte or s = 255 gives NaN.
This test runs that bit arithmetic for all 256 bytes x all 256 scale bytes
and states where it is exact: everywhere the dequantised value is a bf16
(every finite result for s >= 3; for s <= 2 the smallest values fall below
bf16's subnormal step 2^-133 and round there, as bf16 arithmetic does).
The GPU tests check the kernels against this on sampled scales.
"""
import numpy as np

from oracle import moe_ref as O


def decode_bits(byte: np.ndarray) -> np.ndarray:
    """prmt (sign replicated into bits 15..8) -> << 4 -> & 0x87f0, per byte."""
    b = byte.astype(np.uint32)
    lane = b | np.where(b & 0x80, 0xFF00, 0).astype(np.uint32)
    return ((lane << 4) & 0x87F0).astype(np.uint16)


def bf16_mul(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """bf16 x bf16 rounded to nearest even (the product of two 8-bit
    significands is exact in float64, and in float32 wherever it is not
    below float32's subnormal range, which these operands never reach)."""
    p = (O.bf16_to_f32(a_bits).astype(np.float64) * O.bf16_to_f32(b_bits).astype(np.float64))
    with np.errstate(over="ignore"):
        return O.f32_to_bf16(p.astype(np.float32))


def mx_decode_scaled(byte: np.ndarray, s: np.ndarray) -> np.ndarray:
    p = decode_bits(byte)
    nan = ((byte & 0x7F) == 0x7F) | (s == 255)
    s = s.astype(np.int64)
    m1 = np.where(s <= 134, (s + 120) << 7, 0x7F00).astype(np.uint16)
    m2 = np.where(s <= 134, 0x3F80, (s - 7) << 7).astype(np.uint16)  # 0x3f80 = 1.0
    out = bf16_mul(bf16_mul(p, m1), m2)
    return np.where(nan, np.uint16(0x7FC0), out)


def test_decode_is_value_times_2_pow_minus_120():
    b = np.arange(256, dtype=np.uint8)
    finite = (b & 0x7F) != 0x7F
    got = O.bf16_to_f32(decode_bits(b)).astype(np.float64)
    want = O.e4m3_to_f32(b).astype(np.float64) * 2.0 ** -120
    assert np.array_equal(got[finite], want[finite])


def test_every_byte_and_scale():
    b, s = np.meshgrid(np.arange(256, dtype=np.uint8), np.arange(256, dtype=np.uint8),
                       indexing="ij")
    b, s = b.ravel(), s.ravel()
    got = O.bf16_to_f32(mx_decode_scaled(b, s)).astype(np.float64)
    with np.errstate(over="ignore"):
        want = O.e4m3_to_f32(b).astype(np.float64) * np.exp2(s.astype(np.float64) - 127.0)
        want[s == 255] = np.nan
        want[np.abs(want) >= 2.0 ** 128] = np.inf * np.sign(want[np.abs(want) >= 2.0 ** 128])
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    # exact wherever the dequantised value is a bf16 (all of s >= 3)
    rep = O.bf16_to_f32(O.f32_to_bf16(np.where(nan, 0, want).astype(np.float32)))
    exact = ~nan & (rep.astype(np.float64) == np.where(nan, 0, want))
    assert np.array_equal(got[exact], want[exact])
    assert exact[(s >= 3) & (s < 255) & ~nan].all()
    # below bf16's subnormal step (s <= 2 only): off by less than 2^-133
    inexact = ~nan & ~exact
    assert np.all(s[inexact] <= 2)
    assert np.all(np.abs(got[inexact] - want[inexact]) < 2.0 ** -133)
