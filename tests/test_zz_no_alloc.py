"""The allocation-free ConvRot W8A8 linear entry point.

ctu_convrot_w8a8_linear_static_scratch serves callers that cannot call cudaMalloc:
its quantized activation and error word live in a device array inside the library.
It must give the same bf16 output as the regular two-step path
(ctu_convrot_quantize + ctu_int8_linear) -- bit-exact, and never more than one bf16
ulp apart, the tolerance the other GEMM tests use -- on consecutive calls that reuse
the shared array.  This file sorts last so a stop-at-first-failure run has executed
every other test before it.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _ulp(a, b):
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(key(a) - key(b))


def _problem(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 30.0
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 0.009 + 1e-3
    bias = torch.randn((n,), generator=g) * 0.02
    return x.to(torch.bfloat16).cuda(), w.cuda(), w_s.cuda(), bias.cuda()


def _static_scratch_linear(x, w, w_s, bias):
    from comfyui_turing_utils_kernel import _lib

    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.load().ctu_convrot_w8a8_linear_static_scratch(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(w_s.data_ptr()), n,
        ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, n, k,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out


def _two_step_linear(x, w, w_s, bias):
    from comfyui_turing_utils_kernel import _C

    q, s = _C.turing_bf16_int8_convrot_quantize(x, 256, False)
    return _C.turing_int8_linear(q, w, s, w_s, bias)


def test_static_scratch_linear_matches_two_step_path_on_consecutive_calls():
    from comfyui_turing_utils_kernel import _lib

    _lib.device_error(torch.cuda.current_device(), clear=True)
    # Two calls in a row on the shared array: a larger problem, then a smaller one with
    # different K and N, so stale codes or scales from the first call would show.
    for m, k, n, seed in ((257, 1536, 512, 1), (129, 1024, 264, 2)):
        x, w, w_s, bias = _problem(m, k, n, seed)
        got = _static_scratch_linear(x, w, w_s, bias)
        ref = _two_step_linear(x, w, w_s, bias)
        torch.cuda.synchronize()
        g, r = _bits(got), _bits(ref)
        assert _ulp(g, r).max() <= 1
        assert np.array_equal(g, r)
    assert _lib.device_error(torch.cuda.current_device(), clear=True) == 0


def test_static_scratch_linear_rejects_oversized_problems():
    from comfyui_turing_utils_kernel import _lib

    x = torch.zeros((8, 256), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((8, 256), dtype=torch.int8, device="cuda")
    s = torch.ones(8, device="cuda")
    out = torch.empty((8, 8), dtype=torch.bfloat16, device="cuda")
    # m * k beyond the 16 MiB code area (checked before any pointer is touched).
    rc = _lib.load().ctu_convrot_w8a8_linear_static_scratch(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(s.data_ptr()), 8,
        None, ctypes.c_void_p(out.data_ptr()), 32768, 8, 1024, None)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT
    assert "at most" in _lib.load().ctu_last_error().decode()


def test_static_scratch_linear_at_the_exact_limits():
    """m = 65536, k = 256 fills the code area to its last byte and uses every scale
    slot: the output must still equal the two-step path bit for bit, with no kernel
    flag raised.  One more row (m = 65537) must be refused before any launch."""
    from comfyui_turing_utils_kernel import _lib

    dev = torch.cuda.current_device()
    _lib.device_error(dev, clear=True)
    m, k, n = 65536, 256, 16
    x, w, w_s, bias = _problem(m, k, n, 3)
    got = _static_scratch_linear(x, w, w_s, bias)
    ref = _two_step_linear(x, w, w_s, bias)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(got), _bits(ref))
    assert _lib.device_error(dev, clear=True) == 0

    x1 = torch.zeros((m + 1, k), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((m + 1, n), dtype=torch.bfloat16, device="cuda")
    rc = _lib.load().ctu_convrot_w8a8_linear_static_scratch(
        ctypes.c_void_p(x1.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(w_s.data_ptr()), n,
        ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()), m + 1, n, k,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT
    assert "at most" in _lib.load().ctu_last_error().decode()
