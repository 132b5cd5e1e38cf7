"""The CPU oracle reproduces the reference kernels' device outputs (golden vectors).

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs
the reference's own kernels (kernel/csrc/turing/{convrot_quant,w4a8,bf16_epilogue}.cu,
compiled for sm_100a by oracle/Makefile) on a B200.
"""

from pathlib import Path

import numpy as np
import pytest

import convrot_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def _quant_cases():
    data = np.load(GOLDEN / "convrot_quant.npz")
    names = sorted({k.split("__")[0] for k in data.files})
    return data, names


QUANT, QUANT_NAMES = _quant_cases()


def _mode(name):
    if "swiglu" in name:
        return oracle.MODE_SWIGLU
    if name.startswith("gelu"):
        return oracle.MODE_GELU
    return oracle.MODE_PLAIN


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", QUANT_NAMES)
def test_convrot_quantize_matches_reference(name, bits):
    x = QUANT[f"{name}__x"]
    codes, scales = oracle.convrot_quantize(x, bits, _mode(name))
    ref_codes = QUANT[f"{name}__int{bits}_codes"]
    ref_scales = QUANT[f"{name}__int{bits}_scales"]
    assert np.array_equal(codes, ref_codes)
    if _mode(name) == oracle.MODE_SWIGLU:
        # SwiGLU uses expf; glibc's and CUDA's expf may differ by one ulp, which can
        # move the fp32 scale by one ulp while leaving the codes unchanged.
        diff = np.abs(scales.view(np.int32).astype(np.int64) - ref_scales.view(np.int32).astype(np.int64))
        assert diff.max() <= 1
    else:
        assert np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))


GEMM = np.load(GOLDEN / "gemm.npz")
GEMM_KEYS = sorted({k.split("__")[0] for k in GEMM.files if k.startswith("m")})


@pytest.mark.parametrize("key", GEMM_KEYS)
def test_int8_and_w4a8_linear_match_reference(key):
    a, w, w4 = GEMM[f"{key}__a"], GEMM[f"{key}__w"], GEMM[f"{key}__w4_packed"]
    a_s, w_s = GEMM[f"{key}__a_scale"], GEMM[f"{key}__w_scale"]
    bias = GEMM[f"{key}__bias"] if f"{key}__bias" in GEMM.files else None
    assert np.array_equal(oracle.int8_linear(a, w, a_s, w_s, bias), GEMM[f"{key}__int8_linear"])
    assert np.array_equal(oracle.w4a8_linear(a, w4, a_s, w_s, bias), GEMM[f"{key}__w4a8_linear"])


def test_reference_epilogue_fuses_the_bias_add():
    # m64_n128_k256: column j's bias cancels the separately rounded product of row j % 64,
    # so the reference's output there is the product's rounding error (fma) rather than 0.
    key = "m64_n128_k256"
    a, w = GEMM[f"{key}__a"], GEMM[f"{key}__w"]
    a_s, w_s, bias = GEMM[f"{key}__a_scale"], GEMM[f"{key}__w_scale"], GEMM[f"{key}__bias"]
    ref = GEMM[f"{key}__int8_linear"]
    rows, cols = np.arange(128) % 64, np.arange(128)
    separate = oracle.int8_linear(a, w, a_s, w_s, bias, fused=False)
    assert np.all((separate[rows, cols] & 0x7FFF) == 0)
    assert np.count_nonzero(ref[rows, cols] & 0x7FFF) >= 100
    assert np.array_equal(oracle.int8_linear(a, w, a_s, w_s, bias, fused=True), ref)


@pytest.mark.parametrize("tag", ["vec", "scalar"])
def test_dequantize_matches_reference(tag):
    out = oracle.epilogue(GEMM["dequant__acc"], GEMM["dequant__a_scale"], GEMM[f"dequant_{tag}__w_scale"],
                          None, add_zero_bias=False)
    assert np.array_equal(out, GEMM[f"dequant_{tag}__out"])


def test_rotation_is_the_kronecker_radix4_transform():
    m = 0.5 * np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
    r = np.kron(np.kron(np.kron(m, m), m), m)
    assert np.abs(r @ r.T - np.eye(256)).max() == 0.0
    rng = np.random.default_rng(3)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((4, 512)).astype(np.float32))
    y = oracle.rotate(x).astype(np.float64)
    xf = oracle.bf16_bits_to_f32(x).astype(np.float64)
    ref = np.concatenate([xf[:, g * 256:(g + 1) * 256] @ r.T for g in range(2)], axis=1)
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


def test_int4_zero_rows_have_the_reference_scale_floor():
    # kernel/scripts/validate_compatible.py:146-155
    codes, scales = oracle.convrot_quantize(np.zeros((2, 512), np.uint16), 4)
    assert not codes.any()
    assert np.all(scales == np.float32(1.0e-10))


def test_int4_pack_roundtrip():
    rng = np.random.default_rng(0)
    v = rng.integers(-8, 8, size=(5, 64)).astype(np.int8)
    assert np.array_equal(oracle.unpack_int4(oracle.pack_int4(v)), v)


def test_scaled_quantizer_oracle_matches_unscaled_with_own_scales():
    # turing_swiglu_int8_convrot_quantize_scaled with each row's own scale must give the
    # unscaled quantizer's codes (the two reference kernels share the code chain,
    # convrot_quant.cu:138-161 and :475-510), including NaN/inf rows.
    rng = np.random.default_rng(5)
    x = rng.standard_normal((9, 2 * 768)).astype(np.float32)
    xb = oracle.f32_to_bf16_bits(x)
    xb[2, 5] = 0x7FC0
    xb[4, 7] = 0x7F80
    for mode in (oracle.MODE_SWIGLU, oracle.MODE_PLAIN):
        codes, scales = oracle.convrot_quantize(xb, 8, mode)
        assert np.array_equal(oracle.convrot_quantize_scaled(xb, scales, mode), codes)


EXTRAS_PATH = GOLDEN / "extras.npz"


@pytest.mark.skipif(not EXTRAS_PATH.exists(), reason="reference fixtures not generated")
def test_codebook_and_scaled_swiglu_match_reference():
    import sys

    sys.path.insert(0, str(GOLDEN))
    import make_golden

    extras = np.load(EXTRAS_PATH)
    for idx, (m, n, k, gs, _) in enumerate(make_golden.CODEBOOK_CASES):
        a, packed, scale, codebook, a_s, c_s, bias = make_golden.codebook_inputs(m, n, k, gs, 4500 + idx)
        ref = extras[f"codebook_m{m}_n{n}_k{k}_g{gs}__out"]
        assert np.array_equal(oracle.codebook_w4a8_linear(a, packed, a_s, scale, c_s, codebook, bias, gs), ref), idx
    codes = oracle.convrot_quantize_scaled(extras["scaled_swiglu__x"], extras["scaled_swiglu__scales"])
    ref = extras["scaled_swiglu__codes"]
    # expf (glibc vs CUDA) may move a code by one step in rare positions.
    assert np.abs(codes.astype(np.int32) - ref.astype(np.int32)).max() <= 1
    assert (codes != ref).mean() < 1e-3


NORMS_PATH = GOLDEN / "norms.npz"


def _norm_float(a: np.ndarray, code: int) -> np.ndarray:
    import torch

    if code == 2:
        return a.astype(np.float64)
    t = torch.from_numpy(np.ascontiguousarray(a)).view(torch.int16)
    t = t.view(torch.bfloat16 if code == 0 else torch.float16)
    return t.float().numpy().astype(np.float64)


def _norm_nan(a: np.ndarray, code: int) -> np.ndarray:
    if code == 2:
        return np.isnan(a)
    return (a.astype(np.uint32) & 0x7FFF) > (0x7F80 if code == 0 else 0x7C00)


def _assert_norm_close(got, want, code, atol):
    # The oracle's 1/sqrt is correctly rounded; the reference's device rsqrtf is within
    # 2 ulp of it.  Everything else (reduction order, contractions, roundings) is exact.
    gm, wm = _norm_nan(got, code), _norm_nan(want, code)
    assert np.array_equal(gm, wm)
    gf, wf = _norm_float(got, code)[~gm], _norm_float(want, code)[~wm]
    assert np.all(np.abs(gf - wf) <= atol + 1e-6 * np.abs(wf))
    if code != 2:
        assert np.mean(got[~gm] == want[~wm]) >= 0.995


@pytest.mark.skipif(not NORMS_PATH.exists(), reason="norm fixtures not generated")
def test_norm_oracle_matches_reference_kernels():
    z = np.load(NORMS_PATH)
    names = sorted({k.split("__")[0] for k in z.files})
    assert any(n.startswith("rms_") for n in names) and any(n.startswith("ln_") for n in names)
    for name in names:
        meta = [int(v) for v in z[f"{name}__meta"]]
        eps = float(z[f"{name}__eps"][0])
        code = meta[0]
        if name.startswith("rms_"):
            _, rows, hidden, prow, stride, off = meta
            width = 4 if code == 2 else 8
            vec = hidden % width == 0 and stride % width == 0 and off == 0
            got = oracle.segmented_rms_adaln(z[f"{name}__x"], z[f"{name}__weight"], z[f"{name}__scale"],
                                             z[f"{name}__shift"], z[f"{name}__segments"], eps, code, vec,
                                             scale_stride=stride, shift_stride=stride, param_rows=prow)
        else:
            got = oracle.layer_norm_adaln(z[f"{name}__x"], z[f"{name}__scale"], z[f"{name}__shift"], eps, code)
        _assert_norm_close(got, z[f"{name}__out"], code, atol={0: 2**-5, 1: 2**-8, 2: 1e-5}[code])


STAGED_PATH = GOLDEN / "staged.npz"


@pytest.mark.skipif(not STAGED_PATH.exists(), reason="staged fixtures not generated")
def test_staged_quantizer_oracle_matches_reference():
    # The reference's staged SwiGLU / GELU quantizers (convrot_quant.cu:184-358) on
    # special and random rows: codes and scales bit-exact with the staged scale formula.
    z = np.load(STAGED_PATH)
    names = sorted({k.split("__")[0] for k in z.files} - {"scaled_f16"})
    assert names
    for name in names:
        fp16 = name.startswith("f16_")
        mode = oracle.MODE_SWIGLU if "swiglu" in name else oracle.MODE_GELU
        for bits in (8, 4):
            if fp16:
                codes, scales = oracle.convrot_quantize_staged_f16(z[f"{name}__x"], bits=bits, mode=mode)
            else:
                codes, scales = oracle.convrot_quantize(z[f"{name}__x"], bits=bits, mode=mode, staged=True)
            want = z[f"{name}__int{bits}_scales"]
            assert np.array_equal(codes, z[f"{name}__int{bits}_codes"]), (name, bits)
            if mode == oracle.MODE_GELU:
                assert np.array_equal(scales.view(np.uint32), want.view(np.uint32)), (name, bits)
                # The row-buffer formula (absmax / qmax) rounds differently in some rows:
                # the staged ops need their own formula to be bit-exact.
                if not fp16 and bits == 4 and name != "gelu_k256":
                    _, rb = oracle.convrot_quantize(z[f"{name}__x"], bits=bits, mode=mode, staged=False)
                    assert not np.array_equal(rb.view(np.uint32), want.view(np.uint32))
            else:  # glibc's expf vs CUDA's: scales within a few ulps
                ulps = np.abs(scales.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
                assert ulps.max() <= 4, (name, bits)
    # fp16 SwiGLU shard with caller-supplied scales, special scales included.
    codes = oracle.convrot_quantize_scaled_f16(z["scaled_f16__x"], z["scaled_f16__scales"])
    diff = np.abs(codes.astype(np.int32) - z["scaled_f16__codes"].astype(np.int32))
    assert diff.max() <= 1 and np.mean(diff != 0) < 1e-3  # expf: one code step in rare positions

