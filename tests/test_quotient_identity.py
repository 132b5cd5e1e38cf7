"""The quantizer forms bf16(bf16(y) / bf16(scale)) as bf16(bf16(y) * rcp(bf16(scale))).

Both operands carry 8 significant bits, so the exact quotient is never a bf16 rounding
midpoint and stays >= 2^-17 (relative) away from every midpoint, while the product with
the correctly rounded reciprocal is within 2^-23 of it: the bf16 roundings agree.  This
test checks that claim exhaustively over every pair of bf16 significands, across the
binades the int8 quantizer produces (|quotient| <= ~128), with IEEE float32 numpy
arithmetic (the reference divides in fp32: convrot_quant.cu:502-505).
"""

import numpy as np

import convrot_oracle as oracle


def test_reciprocal_product_rounds_like_the_ieee_quotient():
    sig = np.arange(128, dtype=np.uint32)
    # Divisors: every bf16 significand in [1, 2) (the exponent only shifts the quotient).
    s_bits = ((127 << 7) | sig).astype(np.uint16)
    s = oracle.bf16_bits_to_f32(s_bits)
    # Dividends: every bf16 significand over binades 2^-12 .. 2^8, both signs.
    exps = np.arange(127 - 12, 127 + 9, dtype=np.uint32)
    y_bits = ((exps[:, None] << 7) | sig[None, :]).reshape(-1).astype(np.uint16)
    y_bits = np.concatenate([y_bits, y_bits | 0x8000])
    y = oracle.bf16_bits_to_f32(y_bits)
    yy, ss = np.meshgrid(y, s, indexing="ij")
    with np.errstate(all="ignore"):
        quotient = (yy / ss).astype(np.float32)
        rcp = (np.float32(1.0) / s).astype(np.float32)
        product = (yy * rcp[None, :]).astype(np.float32)
    q_ref = oracle.f32_to_bf16_bits(quotient)
    q_fast = oracle.f32_to_bf16_bits(product)
    assert q_ref.size == 2 * len(exps) * 128 * 128
    assert np.array_equal(q_ref, q_fast)
    # And the int8 codes built on them agree as well.
    c_ref = np.clip(np.rint(oracle.bf16_bits_to_f32(q_ref)), -128, 127)
    c_fast = np.clip(np.rint(oracle.bf16_bits_to_f32(q_fast)), -128, 127)
    assert np.array_equal(c_ref, c_fast)
