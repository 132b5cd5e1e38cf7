"""Full-size parity of the two FFN linears of BASELINE configs[1] against the reference's
own kernels on the same GPU.

oracle/_ref/libctu_ref.so is the reference's kernel/csrc/turing/convrot_quant.cu and
w4a8.cu built for sm_100a.  At M = 32760 tokens, FFN up (K = 5120 -> N = 13824) and FFN
down (K = 13824 -> N = 5120) run through every B200 quantizer kernel and both B200 GEMM
kernels on the same inputs as the reference's row-buffer quantizer
(convrot_quant.cu:665-688) and W8A8 GEMM with its dequant + bias epilogue
(w4a8.cu:1185-1219).  Codes, scales and the bf16 outputs must be equal over every row,
not a sample.  The fused tanh-GELU quantizer of the FFN-down input is checked the same
way at full size, against both the reference's row-buffer kernel
(convrot_quant.cu:715-745) and its staged two-kernel path (convrot_quant.cu:184-358).
The W8A8 epilogue is also compared with the reference's at non-finite, overflowing,
subnormal and signed-zero scales and biases, and every quantizer kernel with the
reference's on NaN / inf / subnormal, huge and scale-floor rows.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libctu_ref.so"
M = 32760
QUANT_KERNELS = {"two_pass": 1, "register": 2, "t4": 3, "k8": 4, "g8": 7, "g8_1": 6, "w8": 8}
GEMM_KERNELS = {"single_cta": 1, "cta_pair": 2}

needs_ref = pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    return mg, mg.load_ref()


@pytest.fixture(scope="module")
def K():
    import comfyui_turing_utils_kernel as K
    from comfyui_turing_utils_kernel import _lib

    _lib.device_error(0, clear=True)
    yield K
    assert _lib.device_error(0, clear=True) == 0, "a kernel recorded a bounded-wait timeout"


def _activation(m, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=g, device="cuda")
    idx = torch.randperm(k, generator=g, device="cuda")[: k // 100]
    x[:, idx] *= 30.0
    return x.to(torch.bfloat16)


def _weights(n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    ws = torch.rand((n,), generator=g, device="cuda") * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g, device="cuda") * 0.02
    return w, ws, bias


class _Forced:
    """Force one quantizer / GEMM kernel through the library's test hooks."""

    def __init__(self, quant=0, gemm=0):
        self.quant, self.gemm = quant, gemm

    def __enter__(self):
        from comfyui_turing_utils_kernel import _lib

        assert _lib.load().ctu_debug_set_quant_kernel(self.quant) >= 0
        assert _lib.load().ctu_debug_set_gemm_kernel(self.gemm) >= 0

    def __exit__(self, *exc):
        from comfyui_turing_utils_kernel import _lib

        _lib.load().ctu_debug_set_quant_kernel(0)
        _lib.load().ctu_debug_set_gemm_kernel(0)


def _same_scales(a, b):
    return torch.equal(a.reshape(-1).view(torch.int32), b.reshape(-1).view(torch.int32))


@needs_ref
@pytest.mark.parametrize("k,n", [(5120, 13824), (13824, 5120)], ids=["ffn_up", "ffn_down"])
def test_ffn_linear_full_size_against_reference_kernels(K, ref, k, n):
    mg, lib = ref
    p = mg.p
    x = _activation(M, k, 21 + k)
    w, ws, bias = _weights(n, k, 31 + n)

    ref_codes = torch.empty((M, k), dtype=torch.int8, device="cuda")
    ref_scales = torch.empty((M, 1), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_bf16_convrot_quantize(p(x), p(ref_codes), p(ref_scales), M, k, 8, 0, 1024, mg.stream()))
    for name, sel in QUANT_KERNELS.items():
        with _Forced(quant=sel):
            codes, scales = K.turing_bf16_int8_convrot_quantize(x, 256)
        assert torch.equal(codes, ref_codes), f"{name}: int8 codes differ"
        assert _same_scales(scales, ref_scales), f"{name}: scales differ"
        del codes, scales

    a_scale = ref_scales.view(-1)
    ref_out = torch.empty((M, n), dtype=torch.bfloat16, device="cuda")
    mg.check(lib, lib.ref_int8_linear(p(ref_codes), p(w), p(a_scale), p(ws), p(bias), p(ref_out), M, n, k, 0,
                                      mg.stream()))
    for name, sel in GEMM_KERNELS.items():
        with _Forced(gemm=sel):
            out = K.turing_int8_linear(ref_codes, w, a_scale, ws, bias)
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), f"{name}: bf16 output differs"
        del out

    # The public entry as a caller uses it: default kernels, quantize then GEMM.
    q, s = K.turing_bf16_int8_convrot_quantize(x, 256)
    out = K.turing_int8_linear(q, w, s, ws, bias)
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))


@needs_ref
def test_int4_quantizer_full_size_against_reference_kernel(K, ref):
    mg, lib = ref
    p = mg.p
    k = 13824
    x = _activation(M, k, 41)
    ref_codes = torch.empty((M, k // 2), dtype=torch.int8, device="cuda")
    ref_scales = torch.empty((M, 1), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_bf16_convrot_quantize(p(x), p(ref_codes), p(ref_scales), M, k, 4, 0, 1024, mg.stream()))
    for name, sel in QUANT_KERNELS.items():
        with _Forced(quant=sel):
            codes, scales = K.turing_bf16_int4_convrot_quantize(x, 256)
        assert torch.equal(codes, ref_codes), f"{name}: int4 codes differ"
        assert _same_scales(scales, ref_scales), f"{name}: scales differ"


@needs_ref
def test_gelu_quantizer_full_size_against_reference_kernels(K, ref):
    mg, lib = ref
    p = mg.p
    k = 13824
    x = _activation(M, k, 51)

    ref_codes = torch.empty((M, k), dtype=torch.int8, device="cuda")
    ref_scales = torch.empty((M, 1), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_bf16_gelu_convrot_quantize(p(x), p(ref_codes), p(ref_scales), M, k, 8, 1024, mg.stream()))
    for name, sel in QUANT_KERNELS.items():
        with _Forced(quant=sel):
            codes, scales = K.turing_bf16_gelu_int8_convrot_quantize(x, 256)
        assert torch.equal(codes, ref_codes), f"{name}: GELU int8 codes differ"
        assert _same_scales(scales, ref_scales), f"{name}: GELU scales differ"
        del codes, scales

    # The staged name keeps the staged kernels' scale formula (absmax * 1/127).
    st_codes = torch.empty_like(ref_codes)
    st_scales = torch.empty_like(ref_scales)
    rotated = torch.empty((M, k), dtype=torch.bfloat16, device="cuda")
    partial = torch.empty((M, k // 256), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_staged_convrot_quantize(p(x), p(st_codes), p(st_scales), p(rotated), p(partial), M, k, 8,
                                                  2, 0, mg.stream()))
    del rotated, partial
    codes, scales = K.turing_gelu_int8_convrot_quantize(x, 256)
    assert torch.equal(codes, st_codes), "staged GELU int8 codes differ"
    assert _same_scales(scales, st_scales), "staged GELU scales differ"


@needs_ref
def test_linear_epilogue_extremes_against_reference_kernel(K, ref):
    """Scales and biases at the edges of fp32 -- inf, NaN, 3e38, subnormal, +-0 -- and
    all-zero activation rows (0 x inf): outputs that overflow to inf, become NaN, land
    in the bf16 subnormal range or keep a zero's sign, through both GEMM kernels and the
    reference's W8A8 GEMM (w4a8.cu:1185-1219), bit for bit."""
    mg, lib = ref
    p = mg.p
    m, n, k = 300, 264, 512
    g = torch.Generator(device="cuda").manual_seed(77)
    a = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
    a[20:22] = 0
    w = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    a_scale = torch.rand((m,), generator=g, device="cuda") * 0.02 + 1e-3
    a_scale[5:10] = torch.tensor([1e30, 1e-30, 3e38, 0.0, 1e-40])
    w_scale = torch.rand((n,), generator=g, device="cuda") * 0.009 + 1e-3
    w_scale[:9] = torch.tensor([float("inf"), float("-inf"), float("nan"), 3e38, 1e-38, 1e-41, 0.0, -0.0, 1e20])
    bias = torch.randn((n,), generator=g, device="cuda") * 0.02
    bias[4:6] = 0.0  # outputs of the tiny weight scales stay tiny: bf16 subnormals
    bias[10:16] = torch.tensor([float("nan"), float("inf"), float("-inf"), -0.0, 3e38, -3e38])

    ref_out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    mg.check(lib, lib.ref_int8_linear(p(a), p(w), p(a_scale), p(w_scale), p(bias), p(ref_out), m, n, k, 0,
                                      mg.stream()))
    torch.cuda.synchronize()
    r = ref_out.float()
    assert torch.isinf(r).any() and torch.isnan(r).any()
    assert ((r != 0) & (r.abs() < 2.0 ** -126)).any()  # bf16 subnormal outputs
    for name, sel in GEMM_KERNELS.items():
        with _Forced(gemm=sel):
            out = K.turing_int8_linear(a, w, a_scale, w_scale, bias)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), f"{name}: bf16 output differs"


@needs_ref
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("k", [5120, 13824])
def test_quantizer_edge_rows_against_reference_kernel(K, ref, k, bits):
    """NaN / inf / subnormal / largest-finite rows, rows at 1e30-3e37 and 2^120-2^124, and
    rows whose scale sits at its floor (int8 1e-30, int4 1e-10), through every B200
    quantizer kernel and the reference's row-buffer kernel (convrot_quant.cu:665-713):
    codes and scales bit for bit."""
    from test_gpu_quant_variants import large_rows, special_rows, tiny_rows, to_bf16_tensor

    mg, lib = ref
    p = mg.p
    xb = np.concatenate([special_rows(18, k, seed=k + 1), large_rows(14, k, seed=k + 2), tiny_rows(16, k, seed=k + 3)])
    x = to_bf16_tensor(xb).cuda()
    rows = x.shape[0]
    ref_codes = torch.empty((rows, k if bits == 8 else k // 2), dtype=torch.int8, device="cuda")
    ref_scales = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_bf16_convrot_quantize(p(x), p(ref_codes), p(ref_scales), rows, k, bits, 0, 1024,
                                                mg.stream()))
    quantize = K.turing_bf16_int8_convrot_quantize if bits == 8 else K.turing_bf16_int4_convrot_quantize
    for name, sel in QUANT_KERNELS.items():
        with _Forced(quant=sel):
            codes, scales = quantize(x, 256)
        torch.cuda.synchronize()
        assert torch.equal(codes, ref_codes), f"{name}: codes differ"
        assert _same_scales(scales, ref_scales), f"{name}: scales differ"
