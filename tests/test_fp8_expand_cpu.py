"""CPU check of the E4M3 -> bf16 expansion the FP8 kernel performs (e4m3x2_to_bf16x2 in
flashact_b200/csrc/fa_engine.cuh), restated bit for bit in numpy for all 256 codes: the sign and
the 7 magnitude bits shifted into a bf16 (sign -> bit 15, magnitude -> bits 4..10) encode the
E4M3 value x 2^-120, E4M3 subnormals included (they land on bf16 subnormals the same 2^-120
apart), so one exact multiply by 2^120 (bf16 0x7B80) recovers every code's value."""
import numpy as np
import torch


def _bf16_bits_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def test_all_codes_expand_exactly():
    codes = np.arange(256, dtype=np.uint32)
    # the kernel's prmt puts byte b at bits 8..15 of a 16-bit half: t = b << 8
    t = codes << 8
    bits = ((t >> 4) & 0x07F0) | (t & 0x8000)
    scaled = _bf16_bits_to_f32(bits).astype(np.float64) * 2.0 ** 120  # exact: powers of two
    ref = torch.from_numpy(codes.astype(np.uint8)).view(torch.float8_e4m3fn).float().numpy().astype(np.float64)
    finite = np.isfinite(ref)  # 0x7F / 0xFF are NaN in E4M3 (never produced by the quantiser)
    assert finite.sum() == 254
    np.testing.assert_array_equal(scaled[finite], ref[finite])
    # the products are representable in bf16 (3 mantissa bits), so the bf16 multiply is exact
    as_bf16 = torch.from_numpy(scaled[finite].astype(np.float32)).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(as_bf16, scaled[finite].astype(np.float32))
    # subnormal codes (exponent field 0) are among them: 2^-9 .. 7 x 2^-9
    sub = (codes & 0x78) == 0
    assert np.all(np.abs(scaled[sub & finite]) <= 7 * 2.0 ** -9)
