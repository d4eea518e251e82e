"""The INT4 dequantizer's fast form, checked on the CPU for every fp16 scale it serves: with the scale's
exponent field at least 5, 16 (u - 8) multiplied by scale / 16 (the scale's bits minus 0x1000) rounds to the
same fp16 as (u - 8) * scale, for every nibble u.  numpy's fp16 multiply forms the exact product in fp32 and
rounds once, as the GPU's half multiply and the reference's float product converted to half do."""
import numpy as np


def test_int4_scale_over_16_identity():
    bits = np.arange(65536, dtype=np.uint32)
    exp = (bits >> 10) & 0x1F
    sel = bits[(exp >= 5) & (exp != 31)]
    s = sel.astype(np.uint16).view(np.float16)
    s16 = (sel - 0x1000).astype(np.uint16).view(np.float16)
    np.testing.assert_array_equal(s16.astype(np.float64) * 16, s.astype(np.float64))
    with np.errstate(over="ignore"):
        for u in range(16):
            direct = (np.float32(u - 8) * s.astype(np.float32)).astype(np.float16)
            hi = np.float16(1024 + 16 * u) - np.float16(1152)   # the high half after the bias subtraction
            assert float(hi) == 16 * (u - 8)
            np.testing.assert_array_equal((hi * s16).view(np.uint16), direct.view(np.uint16))
