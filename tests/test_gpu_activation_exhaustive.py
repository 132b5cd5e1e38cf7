"""Every input bit pattern through the fused activations, against the reference kernels.

The fused GELU / SwiGLU quantizers take the activation of one 16-bit input from a table
(per device, filled once).  These tests feed all 65536 bf16 (and, for the staged names,
fp16) patterns through the B200 kernels and through the reference's own kernels
(oracle/_ref, kernel/csrc/turing/convrot_quant.cu built for sm_100a): row r holds
pattern r in column 0 of a single 256-column group and zeros elsewhere, so the row's
scale is |act(pattern)| / 16 / qmax rounded, and its codes carry the sign pattern of the
rotation.  Codes and scales must agree bit for bit for every pattern, on every quantizer
kernel (two-pass, register-resident, four-lane).  SwiGLU rows use up = -1.3 so the
product with the up projection is exercised too (convrot_quant.cu:138-161).
"""

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libctu_ref.so"
KERNELS = {"two_pass": 1, "register": 2, "t4": 3, "k8": 4, "g8": 7, "g8_1": 6, "w8": 8}
ACT_SWIGLU, ACT_GELU = 1, 2


def _ref():
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    return mg, mg.load_ref()


def _rows(dtype: torch.dtype, act: int) -> torch.Tensor:
    patterns = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(dtype)
    x = torch.zeros((65536, 512 if act == ACT_SWIGLU else 256), dtype=dtype)
    x[:, 0] = patterns
    if act == ACT_SWIGLU:
        x[:, 256:] = -1.3
    return x.cuda()


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    view = torch.int32 if a.dtype == torch.float32 else a.dtype
    return torch.equal(a.view(view), b.view(view))


@pytest.fixture(params=list(KERNELS))
def kernel(request):
    from comfyui_turing_utils_kernel import _lib

    assert _lib.load().ctu_debug_set_quant_kernel(KERNELS[request.param]) >= 0
    yield request.param
    _lib.load().ctu_debug_set_quant_kernel(0)


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("act", [ACT_GELU, ACT_SWIGLU])
@pytest.mark.parametrize("bits", [8, 4])
def test_row_buffer_activations_every_bf16_pattern(kernel, act, bits):
    from comfyui_turing_utils_kernel import _C

    mg, lib = _ref()
    x = _rows(torch.bfloat16, act)
    rows = x.shape[0]
    codes = torch.empty((rows, 256 if bits == 8 else 128), dtype=torch.int8, device="cuda")
    scales = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
    if act == ACT_GELU:
        mg.check(lib, lib.ref_bf16_gelu_convrot_quantize(mg.p(x), mg.p(codes), mg.p(scales), rows, 256, bits, 512,
                                                         mg.stream()))
        fn = _C.turing_bf16_gelu_int8_convrot_quantize if bits == 8 else _C.turing_bf16_gelu_int4_convrot_quantize
        got_codes, got_scales = fn(x, 256)
    else:
        mg.check(lib, lib.ref_bf16_convrot_quantize(mg.p(x), mg.p(codes), mg.p(scales), rows, 256, bits, 1, 512,
                                                    mg.stream()))
        fn = _C.turing_bf16_int8_convrot_quantize if bits == 8 else _C.turing_bf16_int4_convrot_quantize
        got_codes, got_scales = fn(x, 256, swiglu=True)
    torch.cuda.synchronize()
    assert _same(got_scales, scales)
    assert torch.equal(got_codes, codes)


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("act", [ACT_GELU, ACT_SWIGLU])
def test_staged_activations_every_pattern(dtype, act):
    # The staged names (convrot_quant.cu:184-358): bf16 and fp16 rows, int8 codes.
    from comfyui_turing_utils_kernel import _C

    mg, lib = _ref()
    x = _rows(dtype, act)
    rows = x.shape[0]
    codes = torch.empty((rows, 256), dtype=torch.int8, device="cuda")
    scales = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
    rotated = torch.empty((rows, 256), dtype=dtype, device="cuda")
    partial = torch.empty((rows, 1), dtype=torch.float32, device="cuda")
    mg.check(lib, lib.ref_staged_convrot_quantize(mg.p(x), mg.p(codes), mg.p(scales), mg.p(rotated), mg.p(partial),
                                                  rows, 256, 8, act, 1 if dtype == torch.float16 else 0,
                                                  mg.stream()))
    fn = _C.turing_gelu_int8_convrot_quantize if act == ACT_GELU else _C.turing_swiglu_int8_convrot_quantize
    got_codes, got_scales = fn(x, 256)
    torch.cuda.synchronize()
    assert _same(got_scales, scales)
    assert torch.equal(got_codes, codes)
