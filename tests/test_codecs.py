"""Exhaustive codec tables (CPU): the oracle's bit-field decoders against torch's
own low-precision dtypes and the reference's tables.

Reference: h4mv/h4mv_test.py:16-17 (E2M1 table), h4mv/h4mv.cu:33-41 (e2m1 bit
rules), h4mv/h4mv.cu:72 (e8m0 as fp32 bits b << 23), vllm-fp8kv/fp8kv_v3.py:61-63
(fp8 e4m3 -> bf16 cast is exact).
"""
import math

import numpy as np
import torch

import fp8kv_oracle as FO
import mxfp4_oracle as MO


def test_e4m3_table_matches_torch():
    ours = FO.e4m3_table()
    codes = torch.arange(256, dtype=torch.uint8)
    theirs = codes.view(torch.float8_e4m3fn).float().numpy()
    nan_o, nan_t = np.isnan(ours), np.isnan(theirs)
    assert (nan_o == nan_t).all()
    assert nan_o.sum() == 2  # 0x7F and 0xFF
    np.testing.assert_array_equal(ours[~nan_o], theirs[~nan_t])
    # e4m3 -> bf16 is exact (every finite code survives a round trip)
    fin = codes[~torch.from_numpy(nan_o)]
    bf = fin.view(torch.float8_e4m3fn).to(torch.bfloat16).float()
    np.testing.assert_array_equal(bf.numpy(), ours[~nan_o])


def test_e4m3_f16_exact():
    codes = torch.arange(256, dtype=torch.uint8)
    f = codes.view(torch.float8_e4m3fn).float()
    fin = ~torch.isnan(f)
    assert torch.equal(f[fin].to(torch.float16).float(), f[fin])


def test_e2m1_bit_rules_match_lut():
    for c in range(16):
        v = MO.e2m1_decode_bits(c)
        ref = MO.E2M1_LUT[c]
        assert v == ref and math.copysign(1.0, v) == math.copysign(1.0, ref), c
    # zero iff (v & 7) == 0 ; 0b1000 is -0 (docs/06-w4gemm-hip-roadmap.md:39-40)
    assert [c for c in range(16) if MO.e2m1_decode_bits(c) == 0] == [0, 8]
    assert MO.e2m1_decode_bits(1) == 0.5 and MO.e2m1_decode_bits(9) == -0.5


def test_e8m0_kernel_semantics():
    b = np.arange(256)
    bits = MO.e8m0_bits(b)
    exp2 = MO.e8m0_exp2(b)
    assert bits[0] == 0.0                      # reference kernel: scale 0
    assert np.isinf(bits[255]) and np.isinf(exp2[255])
    np.testing.assert_array_equal(bits[1:255], exp2[1:255])
    # torch's e8m0 agrees on the normal range
    t = torch.arange(1, 255, dtype=torch.uint8).view(torch.float8_e8m0fnu).float().numpy()
    np.testing.assert_array_equal(t, exp2[1:255])


def test_bf16_lowexp_construction_is_exact():
    """The GEMV dequant builds bf16 bits (sign << 15) | (mag << 6), i.e. the e2m1
    value times 2^-126, then multiplies by 2^(s-1).  Check the algebra on CPU
    for every code and every scale byte (bf16 subnormals included)."""
    codes = np.arange(16, dtype=np.uint32)
    raw = ((codes >> 3) << 15) | ((codes & 7) << 6)
    low = torch.from_numpy(raw.astype(np.int32)).to(torch.int16).view(torch.bfloat16).double()
    lut = torch.tensor(MO.E2M1_LUT, dtype=torch.float64)
    assert torch.equal(low * 2.0 ** 126, lut)
    for s in range(0, 256):
        scale = float(MO.e8m0_bits(s))
        want = lut * scale if s not in (0, 255) else None
        if s == 0:
            m1 = 0.0
            got = low * m1
            assert torch.all(got == 0)
        elif s <= 128:
            got = (low * 2.0 ** (s - 1)).to(torch.bfloat16).double()
            assert torch.equal(got, want), s
        elif s < 255:
            got = ((low * 2.0 ** 126).to(torch.bfloat16).double() * 2.0 ** (s - 127)).to(torch.bfloat16).double()
            # values beyond the bf16 range become inf, as the fp32 path of the reference would
            assert torch.equal(got, want.to(torch.bfloat16).double()), s
