"""The ConvRot quantizer kernels -- two-pass (bf16(y) back to shared memory, then a
quantize pass), register-resident (two lanes per group, whole rows per batch, codes from
registers), four-lane and eight-lane transpose (stages 3-4 after a shared-memory
transpose) -- against the reference's golden vectors and the oracle.

The library picks a kernel per width; ``ctu_debug_set_quant_kernel`` forces one kernel
so every kernel is checked on every case.
"""

import numpy as np
import pytest
import torch

import convrot_oracle as oracle

pytestmark = pytest.mark.gpu

from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"
QUANT = np.load(GOLDEN / "convrot_quant.npz")
QUANT_NAMES = sorted({k.split("__")[0] for k in QUANT.files})
KERNELS = {"two_pass": 1, "register": 2, "t4": 3, "k8": 4, "g8": 7, "g8_1": 6, "w8": 8}


@pytest.fixture(scope="module")
def C():
    from comfyui_turing_utils_kernel import _C, _lib

    _lib.device_error(0, clear=True)
    yield _C
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


@pytest.fixture(params=list(KERNELS))
def kernel(request):
    from comfyui_turing_utils_kernel import _lib

    prev = _lib.load().ctu_debug_set_quant_kernel(KERNELS[request.param])
    assert prev >= 0
    yield request.param
    _lib.load().ctu_debug_set_quant_kernel(0)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def activations(rows, width, seed, outlier_scale=30.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, width), generator=g)
    idx = torch.randperm(width, generator=g)[: max(1, width // 100)]
    x[:, idx] *= outlier_scale
    return x.to(torch.bfloat16)


def run_quant(C, x_bits, bits, mode="plain"):
    x = to_bf16_tensor(x_bits).cuda()
    if mode == "gelu":
        fn = C.turing_bf16_gelu_int8_convrot_quantize if bits == 8 else C.turing_bf16_gelu_int4_convrot_quantize
        codes, scales = fn(x, 256)
    else:
        fn = C.turing_bf16_int8_convrot_quantize if bits == 8 else C.turing_bf16_int4_convrot_quantize
        codes, scales = fn(x, 256, mode == "swiglu")
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy().reshape(-1)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", QUANT_NAMES)
def test_golden(C, kernel, name, bits):
    mode = "swiglu" if "swiglu" in name else ("gelu" if name.startswith("gelu") else "plain")
    codes, scales = run_quant(C, QUANT[f"{name}__x"], bits, mode)
    assert np.array_equal(codes, QUANT[f"{name}__int{bits}_codes"])
    assert np.array_equal(scales.view(np.uint32), QUANT[f"{name}__int{bits}_scales"].view(np.uint32))


# Widths on both sides of every batch plan (one row per batch at 54 groups, several
# rows at 6 or 20 groups, the register kernel's 128-group limit) and row counts that
# leave partial last batches.
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(1, 256), (3, 512), (17, 1536), (33, 5120), (5, 13824), (130, 768),
                                    (7, 2560), (64, 1024), (2, 16384), (3, 32768), (2, 33024), (61, 4096),
                                    (257, 3072), (1000, 5120)])
def test_oracle(C, kernel, rows, k, bits):
    x = activations(rows, k, seed=rows * 131 + k)
    xb = bf16_bits(x)
    codes, scales = run_quant(C, xb, bits)
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits)
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


def special_rows(rows, k, seed):
    """bf16 rows mixing NaN, +-inf, subnormals, +-0, the largest finite values and
    ordinary activations, one kind of trouble per row and some rows clean."""
    rng = np.random.default_rng(seed)
    x = bf16_bits(activations(rows, k, seed))
    specials = [0x7FC0, 0xFFC0, 0x7F80, 0xFF80, 0x0001, 0x8001, 0x007F, 0x0000, 0x8000, 0x7F7F, 0xFF7F]
    for r in range(rows):
        kind = r % 6
        cols = rng.choice(k, size=max(1, k // 64), replace=False)
        if kind == 0:
            x[r, cols] = rng.choice(specials, size=cols.size)
        elif kind == 1:
            x[r, cols] = 0x7F7F  # many maxima: sums overflow to inf
        elif kind == 2:
            x[r, :] = rng.choice([0x0001, 0x8001, 0x0003, 0x0000], size=k)  # all subnormal
        elif kind == 3:
            x[r, cols[:1]] = 0x7FC0  # a single NaN
        elif kind == 4:
            x[r, cols[:2]] = [0x7F80, 0xFF80]  # +inf and -inf: NaN after the rotation
    return x


def large_rows(rows, k, seed):
    """Rows scaled to magnitudes where the kernels' scaling shortcuts meet their limits:
    1e31 and 1e36 (the int4 reciprocal falls below 2^-100; the rotation stays finite
    without its halvings), 2^120 to 2^124 (finite in the reference's order, overflowing
    without the halvings), and rows mixing such groups with ordinary ones."""
    x = activations(rows, k, seed).float()
    mags = [1e31, 1e36, 2.0 ** 120, 2.0 ** 122, 2.0 ** 124, 1e30, 3e37]
    for r in range(rows):
        m = mags[r % len(mags)]
        if r % 2 == 0:
            x[r] = x[r] / x[r].abs().max() * m
        else:  # only the first group of the row is large
            x[r, :256] = x[r, :256] / x[r, :256].abs().max() * m
    return bf16_bits(x.to(torch.bfloat16))


def tiny_rows(rows, k, seed):
    """Rows small enough that the scale's floor decides it (int8: 1e-30, so a row absmax
    below 127e-30; int4: 1e-10, below 7e-10) while their codes are still non-zero, and
    rows mixing one such group with ordinary ones.  All values stay normal bf16."""
    x = activations(rows, k, seed).float()
    mags = [1e-28, 1e-29, 5e-29, 3e-31, 5e-10, 1e-36, 3e-10, 3e-11]
    for r in range(rows):
        m = mags[r % len(mags)]
        if r % 2 == 0:
            x[r] = x[r] / x[r].abs().max() * m
        else:  # only the first group of the row is tiny
            x[r, :256] = x[r, :256] / x[r, :256].abs().max() * m
    return bf16_bits(x.to(torch.bfloat16))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(16, 512), (16, 5120), (8, 13824)])
def test_scale_floor_rows(C, kernel, rows, k, bits):
    xb = tiny_rows(rows, k, seed=rows * 5 + k)
    codes, scales = run_quant(C, xb, bits)
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits)
    assert np.count_nonzero(ref_codes[0::2]) > 0  # floored rows with non-zero codes
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(14, 512), (14, 5120), (7, 13824)])
def test_large_magnitudes(C, kernel, rows, k, bits):
    xb = large_rows(rows, k, seed=rows * 3 + k)
    codes, scales = run_quant(C, xb, bits)
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits)
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,k", [(12, 512), (18, 5120), (7, 13824)])
def test_special_values(C, kernel, rows, k, bits):
    xb = special_rows(rows, k, seed=rows + k)
    codes, scales = run_quant(C, xb, bits)
    ref_codes, ref_scales = oracle.convrot_quantize(xb, bits)
    assert np.array_equal(codes, ref_codes)
    assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("mode", ["swiglu", "gelu"])
def test_fused_activations_against_each_other(C, mode, bits):
    # The two kernels share the activation code: their outputs must be identical.
    from comfyui_turing_utils_kernel import _lib

    width = 2 * 5120 if mode == "swiglu" else 5120
    xb = bf16_bits(activations(37, width, seed=77))
    out = {}
    try:
        for name, sel in KERNELS.items():
            _lib.load().ctu_debug_set_quant_kernel(sel)
            out[name] = run_quant(C, xb, bits, mode)
    finally:
        _lib.load().ctu_debug_set_quant_kernel(0)
    for name in [n for n in KERNELS if n != "two_pass"]:
        assert np.array_equal(out["two_pass"][0], out[name][0])
        assert np.array_equal(out["two_pass"][1].view(np.uint32), out[name][1].view(np.uint32))


def test_full_size_kernels_agree(C):
    # Wan-14B activation shapes: both kernels give identical codes and scales.
    from comfyui_turing_utils_kernel import _lib

    for k in (5120, 13824):
        x = activations(32760, k, seed=k).cuda()
        res = {}
        try:
            for name, sel in KERNELS.items():
                _lib.load().ctu_debug_set_quant_kernel(sel)
                res[name] = C.turing_bf16_int8_convrot_quantize(x, 256, False)
        finally:
            _lib.load().ctu_debug_set_quant_kernel(0)
        torch.cuda.synchronize()
        for name in [n for n in KERNELS if n != "two_pass"]:
            assert torch.equal(res["two_pass"][0], res[name][0])
            assert torch.equal(res["two_pass"][1], res[name][1])


# ----------------------------------------------------------------------------- scaled SwiGLU shards
def test_scaled_swiglu_shards_reassemble_the_row(C, kernel):
    # Exact two-pass channel streaming (dispatch.py:67-69): whole-row scales from the
    # unscaled op, then each 256-aligned channel shard quantized with them, must give
    # the unscaled op's codes.
    rows, k, shards = 37, 5120, 4
    xb = bf16_bits(activations(rows, 2 * k, seed=91))
    x = to_bf16_tensor(xb).cuda()
    codes, scales = C.turing_bf16_int8_convrot_quantize(x, 256, True)
    width = k // shards
    parts = []
    for j in range(shards):
        gate = x[:, j * width:(j + 1) * width]
        up = x[:, k + j * width:k + (j + 1) * width]
        parts.append(C.turing_swiglu_int8_convrot_quantize_scaled(torch.cat([gate, up], dim=1), scales, 256))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts, dim=1), codes)


@pytest.mark.parametrize("rows,k", [(5, 512), (19, 5120), (3, 13824)])
def test_scaled_swiglu_matches_oracle_with_any_scale(C, kernel, rows, k):
    rng = np.random.default_rng(rows + k)
    xb = bf16_bits(activations(rows, 2 * k, seed=rows * 7 + k))
    if rows > 4:
        xb[1, rng.choice(2 * k, size=3, replace=False)] = [0x7FC0, 0x7F80, 0xFF80]  # NaN and infinities
    scales = (rng.random(rows).astype(np.float32) * 0.05 + 1e-3)
    specials = np.array([0.0, np.nan, np.inf, -0.03, 1e-40, 3e38], dtype=np.float32)
    scales[: min(rows, specials.size)] = specials[: min(rows, specials.size)]
    codes = C.turing_swiglu_int8_convrot_quantize_scaled(to_bf16_tensor(xb).cuda(), torch.from_numpy(scales).cuda(), 256)
    torch.cuda.synchronize()
    ref = oracle.convrot_quantize_scaled(xb, scales)
    got = codes.cpu().numpy()
    # SwiGLU uses expf: CUDA and glibc may differ by one ulp, which can move a code by
    # one step in rare positions (same tolerance as the unscaled SwiGLU test).
    assert np.abs(got.astype(np.int32) - ref.astype(np.int32)).max() <= 1
    assert (got != ref).mean() < 1e-3


def test_scaled_swiglu_rejects_bad_scales(C):
    x = torch.zeros((4, 1024), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="one FP32 scale per input row"):
        C.turing_swiglu_int8_convrot_quantize_scaled(x, torch.ones(3, device="cuda"), 256)
    with pytest.raises(RuntimeError, match="group_size=256"):
        C.turing_swiglu_int8_convrot_quantize_scaled(x, torch.ones(4, device="cuda"), 128)


# ----------------------------------------------------------------------------- staged op names
STAGED_PATH = Path(__file__).resolve().parent / "golden" / "staged.npz"


@pytest.mark.skipif(not STAGED_PATH.exists(), reason="staged fixtures not generated")
def test_staged_ops_match_reference_staged_kernels(C, kernel):
    # turing_swiglu_int{8,4}_convrot_quantize / turing_gelu_int{8,4}_convrot_quantize keep the
    # staged kernels' scale formula (absmax * (1/qmax)); bit-exact against those kernels.
    z = np.load(STAGED_PATH)
    for name in sorted({k.split("__")[0] for k in z.files} - {"scaled_f16"}):
        fp16 = name.startswith("f16_")
        x = torch.from_numpy(z[f"{name}__x"].astype(np.int16)).view(torch.float16 if fp16 else torch.bfloat16).cuda()
        act = "swiglu" if "swiglu" in name else "gelu"
        for bits in (8, 4):
            fn = getattr(C, f"turing_{act}_int{bits}_convrot_quantize")
            codes, scales = fn(x, 256)
            torch.cuda.synchronize()
            assert np.array_equal(codes.cpu().numpy(), z[f"{name}__int{bits}_codes"]), (name, bits)
            assert np.array_equal(scales.cpu().numpy().reshape(-1).view(np.uint32),
                                  z[f"{name}__int{bits}_scales"].view(np.uint32)), (name, bits)


@pytest.mark.parametrize("act,k", [("swiglu", 5120), ("gelu", 1536), ("gelu", 13824)])
def test_staged_ops_match_oracle(C, kernel, act, k):
    # The oracle evaluates expf / tanhf with the host's libm, which may differ from CUDA's
    # by one ulp; the scale then differs by an ulp or so and a rare code by one step
    # (the reference fixtures above pin the device results exactly).
    rows = 300
    width = 2 * k if act == "swiglu" else k
    g = torch.Generator().manual_seed(k + rows)
    x = (torch.randn((rows, width), generator=g) * 3).to(torch.bfloat16)
    bits_x = x.view(torch.int16).numpy().view(np.uint16)
    mode = oracle.MODE_SWIGLU if act == "swiglu" else oracle.MODE_GELU
    for bits in (8, 4):
        codes, scales = getattr(C, f"turing_{act}_int{bits}_convrot_quantize")(x.cuda(), 256)
        torch.cuda.synchronize()
        want_codes, want_scales = oracle.convrot_quantize(bits_x, bits=bits, mode=mode, staged=True)
        got_s = scales.cpu().numpy().reshape(-1)
        ulps = np.abs(got_s.view(np.int32).astype(np.int64) - want_scales.view(np.int32).astype(np.int64))
        if act == "swiglu":  # expf feeds the product directly: a few ulps in some rows
            assert ulps.max() <= 8 and np.mean(ulps == 0) > 0.8
        else:
            assert ulps.max() <= 2 and np.mean(ulps == 0) > 0.9
        got = codes.cpu().numpy()
        if bits == 4:
            got, want = oracle.unpack_int4(got), oracle.unpack_int4(want_codes)
        else:
            want = want_codes
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1 and np.mean(diff != 0) < (1e-2 if act == "swiglu" else 1e-3)


@pytest.mark.skipif(not STAGED_PATH.exists(), reason="staged fixtures not generated")
def test_scaled_swiglu_fp16_matches_reference(C):
    z = np.load(STAGED_PATH)
    x = torch.from_numpy(z["scaled_f16__x"].astype(np.int16)).view(torch.float16).cuda()
    codes = C.turing_swiglu_int8_convrot_quantize_scaled(x, torch.from_numpy(z["scaled_f16__scales"]).cuda(), 256)
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), z["scaled_f16__codes"])


def test_row_buffer_names_reject_fp16(C):
    x = torch.zeros((4, 512), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="bfloat16"):
        C.turing_bf16_int8_convrot_quantize(x, 256)
    with pytest.raises(RuntimeError, match="bfloat16"):
        C.turing_bf16_gelu_int8_convrot_quantize(x, 256)

