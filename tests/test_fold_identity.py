"""The arithmetic the warp-row and multi-group quantizers use for bf16-valued rows
(plain rows, tanh-GELU table values), checked on the CPU with IEEE float32 numpy.

1. Folded halvings: the reference's four radix-4 stages (convrot_quant.cu:104-116, each
   output 0.5 * (((x0 +- x1) +- x2) +- x3)) without the four multiplications by 0.5 give
   z = 16 y exactly, bit for bit, whenever z is finite.  (Every bf16 value is a multiple
   of 2^-133, so every intermediate is a multiple of 2^-137: no halving rounds, and
   rounding commutes with the power-of-two scaling.)
2. The code chains built on it: the int8 codes from bf16(z) * (rcp(bf16(scale)) / 16) and
   the int4 codes from bf16(z) * (1/scale / 16) -- or, when 1/scale < 2^-100,
   (bf16(z) / 16) * (1/scale) -- equal the reference's codes from bf16(y)
   (convrot_quant.cu:475-510; the oracle restates them).
"""

import numpy as np

import convrot_oracle as oracle

F32 = np.float32
HALF = F32(0.5)


def _stage_indices(stride):
    lane = np.arange(64)
    base = lane % stride + (lane // stride) * (4 * stride)
    return base, base + stride, base + 2 * stride, base + 3 * stride


STAGES = [_stage_indices(s) for s in (1, 4, 16, 64)]


def rotate(groups: np.ndarray, halve: bool) -> np.ndarray:
    """The four radix-4 stages over [G, 256] float32 groups, in the reference's order of
    operations; `halve=False` drops the per-stage multiplication by 0.5."""
    v = groups.astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        for i0, i1, i2, i3 in STAGES:
            x0, x1, x2, x3 = v[:, i0], v[:, i1], v[:, i2], v[:, i3]
            out = np.empty_like(v)
            out[:, i0] = ((x0 + x1) + x2) - x3
            out[:, i1] = ((x0 + x1) - x2) + x3
            out[:, i2] = ((x0 - x1) + x2) + x3
            out[:, i3] = ((-x0 + x1) + x2) + x3
            if halve:
                out *= HALF
            v = out
    return v


def bf16_values(bits: np.ndarray) -> np.ndarray:
    return oracle.bf16_bits_to_f32(np.asarray(bits, dtype=np.uint16))


def random_finite_bf16(rng, shape):
    """Random bf16 bit patterns over every finite exponent (subnormals included)."""
    bits = rng.integers(0, 1 << 16, size=shape, dtype=np.uint32).astype(np.uint16)
    exp = (bits >> 7) & 0xFF
    return np.where(exp == 0xFF, bits & 0x807F, bits).astype(np.uint16)  # inf/NaN -> exponent 0


def scaled_groups(rng, n, mags):
    """N(0, 1) groups, each rescaled so its largest magnitude is one of `mags`, rounded to bf16."""
    x = rng.standard_normal((n, 256)).astype(np.float32)
    m = np.asarray(mags, dtype=np.float64)[rng.integers(0, len(mags), size=n)]
    x = (x / np.abs(x).max(axis=1, keepdims=True) * m[:, None]).astype(np.float32)
    return oracle.f32_to_bf16_bits(x)


def check_fold(bits):
    x = bf16_values(bits).reshape(-1, 256)
    y = rotate(x, halve=True)
    z = rotate(x, halve=False)
    finite = np.isfinite(z).all(axis=1)
    assert finite.any()
    with np.errstate(over="ignore"):
        y16 = (y[finite] * F32(16.0)).astype(np.float32)
    assert np.array_equal(z[finite].view(np.uint32), y16.view(np.uint32))
    return finite


def test_rotation_emulation_matches_the_oracle():
    rng = np.random.default_rng(1)
    bits = scaled_groups(rng, 64, [1.0, 30.0, 1e-20, 1e20]).reshape(4, -1)  # rows of 16 groups
    y = oracle.rotate(bits)
    assert np.array_equal(rotate(bf16_values(bits).reshape(-1, 256), True).reshape(y.shape).view(np.uint32),
                          y.view(np.uint32))


def test_folded_rotation_is_sixteen_times_the_reference():
    rng = np.random.default_rng(2)
    # Random bit patterns over every finite exponent: huge, ordinary, tiny and subnormal
    # values side by side in one group.
    check_fold(random_finite_bf16(rng, (20000, 256)))
    # Groups confined to one magnitude, from the subnormal range to just below overflow.
    mags = [2.0 ** -133 * 3, 1e-39, 2.0 ** -126, 1e-30, 1e-10, 1.0, 1e10, 1e30, 2.0 ** 120, 3e37]
    finite = check_fold(scaled_groups(rng, 20000, mags))
    # Groups near the top of the range overflow without the halvings (the kernels
    # recompute those in the reference's order); the rest are all folded.
    assert 0 < np.count_nonzero(~finite) < finite.size


def _rows(rng, rows, groups, mags):
    return scaled_groups(rng, rows * groups, mags).reshape(rows, groups * 256)


def test_folded_int8_and_int4_code_chains_match_the_reference():
    rng = np.random.default_rng(3)
    mags = [1e-36, 3e-31, 5e-29, 1e-28, 3e-11, 3e-10, 5e-10, 1e-3, 1.0, 30.0, 1e10, 1e30, 1e36]
    for groups in (1, 5):
        bits = _rows(rng, 400, groups, mags)
        rows, k = bits.shape
        x = bf16_values(bits).reshape(-1, 256)
        y = rotate(x, halve=True).reshape(rows, k)
        z = rotate(x, halve=False).reshape(rows, k)
        keep = np.isfinite(z).all(axis=1) & np.isfinite(y).all(axis=1)  # every group folded
        wz = bf16_values(oracle.f32_to_bf16_bits(z))  # the kernels' rotated words, bf16(z)

        ref8, scale8 = oracle.convrot_quantize(bits, 8)
        rs = bf16_values(oracle.f32_to_bf16_bits(scale8))
        rc = ((F32(1.0) / rs).astype(np.float32) * F32(0.0625)).astype(np.float32)
        with np.errstate(over="ignore", invalid="ignore"):
            q = bf16_values(oracle.f32_to_bf16_bits((wz * rc[:, None]).astype(np.float32)))
        codes8 = np.clip(np.rint(q), -128, 127).astype(np.int8)
        assert keep.sum() > rows // 2
        assert np.array_equal(codes8[keep], ref8[keep])

        ref4, scale4 = oracle.convrot_quantize(bits, 4)
        inv = (F32(1.0) / scale4).astype(np.float32)
        with np.errstate(over="ignore", invalid="ignore"):
            pre = ((wz * F32(0.0625)).astype(np.float32) * inv[:, None]).astype(np.float32)
            post = (wz * (inv * F32(0.0625)).astype(np.float32)[:, None]).astype(np.float32)
        p = np.where((inv >= F32(2.0 ** -100))[:, None], post, pre)
        c4 = np.clip(np.rint(p), -7, 7).astype(np.int8)
        packed = ((c4[:, 0::2] & 0x0F) | ((c4[:, 1::2] & 0x0F) << 4)).astype(np.uint8).view(np.int8)
        assert np.array_equal(packed[keep], ref4[keep])
