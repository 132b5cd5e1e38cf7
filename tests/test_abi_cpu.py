"""CPU-side checks of the C ABI library and the drop-in Python surface (no GPU calls)."""

import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "ctu_b200.h").read_text()
    return sorted(set(re.findall(r"CTU_API\s+(?:const\s+)?\w+\s*\*?\s*(ctu_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 7
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"
    assert lib.ctu_version() >= (0 << 16) | (1 << 8)


def test_argument_errors_are_reported_without_a_gpu():
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    rc = lib.ctu_convrot_quantize(null, 4, 300, 0, 8, null, null, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT
    assert "divisible by 256" in lib.ctu_last_error().decode()
    rc = lib.ctu_int8_linear(null, null, null, null, 8, null, null, 4, 8, 24, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT
    assert "K%16=0" in lib.ctu_last_error().decode()
    rc = lib.ctu_convrot_quantize(null, 0, 512, 0, 8, null, null, null)
    assert rc == _lib.CTU_OK  # empty batch is a no-op


def test_reference_c_module_attribute_names():
    # Names probed by the plugin through kernel_extension_has_symbol (kernel_api.py:26-37).
    from comfyui_turing_utils_kernel import _C

    for name in ("turing_int8_linear", "turing_w4a8_linear", "turing_dequantize_int8_bf16", "turing_bf16_int8_convrot_quantize",
                 "turing_bf16_int4_convrot_quantize", "turing_bf16_gelu_int8_convrot_quantize",
                 "turing_bf16_gelu_int4_convrot_quantize", "turing_swiglu_int8_convrot_quantize",
                 "turing_swiglu_int4_convrot_quantize", "turing_gelu_int8_convrot_quantize",
                 "turing_gelu_int4_convrot_quantize"):
        assert callable(getattr(_C, name)), name


def test_custom_op_fake_shapes():
    # kernel tests/test_kernel_custom_ops.py:515-607 of the reference: meta shapes.
    import comfyui_turing_utils_kernel as k

    x = torch.empty((3, 512), dtype=torch.bfloat16, device="meta")
    q, s = k.turing_bf16_int8_convrot_quantize(x, 256, swiglu=True)
    assert q.shape == (3, 256) and q.dtype == torch.int8 and s.shape == (3, 1) and s.dtype == torch.float32
    q, s = k.turing_bf16_int4_convrot_quantize(x, 256, swiglu=True)
    assert q.shape == (3, 128)
    q, s = k.turing_bf16_int4_convrot_quantize(x, 256)
    assert q.shape == (3, 256)
    q, s = k.turing_bf16_gelu_int8_convrot_quantize(x, 256)
    assert q.shape == (3, 512)
    a = torch.empty((7, 64), dtype=torch.int8, device="meta")
    w = torch.empty((16, 64), dtype=torch.int8, device="meta")
    out = k.turing_int8_linear(a, w, torch.empty(7, device="meta"), torch.empty(16, device="meta"))
    assert out.shape == (7, 16) and out.dtype == torch.bfloat16
    acc = torch.empty((5, 24), dtype=torch.int32, device="meta")
    assert k.turing_dequantize_int8_bf16(acc, torch.empty(5, device="meta"), torch.empty(1, device="meta"),
                                         16).shape == (5, 16)


def test_ops_refuse_cpu_tensors():
    import comfyui_turing_utils_kernel as k

    with pytest.raises(RuntimeError, match="CUDA"):
        k.turing_bf16_int8_convrot_quantize(torch.zeros((2, 256), dtype=torch.bfloat16), 256)


def test_quantizer_selection_per_width():
    # The per-width choice the measurements in the kernel sources justify, evaluated on the
    # host for B200's 227 KB of opt-in shared memory: the multi-group eight-lane kernel for
    # plain and GELU rows wider than 4096 (one group per team at K = 5120, two at K = 13824),
    # eight lanes for SwiGLU at K = 5120, four lanes at K <= 4096, and the two-pass kernel
    # beyond K = 32768.
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    two_pass, reg, t4, k8, g8 = 0, 1, 2, 3, 4

    def plan(k, act=0, bits=8):
        kind, warps, rows = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        rc = lib.ctu_debug_quant_plan(k, act, bits, 232448, ctypes.byref(kind), ctypes.byref(warps), ctypes.byref(rows))
        assert rc == 0, lib.ctu_last_error().decode()
        return kind.value, warps.value, rows.value

    assert plan(5120) == (g8, 5, 1)
    assert plan(5120, act=2)[0] == g8 and plan(5120, bits=4)[0] == g8
    assert plan(5120, act=1)[0] == k8
    for k in (256, 1536, 3072, 4096):
        assert plan(k)[0] == t4, k
    assert plan(13824) == (g8, 7, 1) and plan(13824, act=2)[0] == g8
    assert plan(13824, act=1)[0] == reg
    assert plan(33024)[0] == two_pass
    # The selector hook forces one kernel wherever the width allows it.
    prev = lib.ctu_debug_set_quant_kernel(2)
    try:
        assert plan(5120)[0] == reg
    finally:
        lib.ctu_debug_set_quant_kernel(prev)
    assert lib.ctu_debug_quant_plan(300, 0, 8, 232448, ctypes.byref(ctypes.c_int()), ctypes.byref(ctypes.c_int()),
                                    ctypes.byref(ctypes.c_int())) == _lib.CTU_ERR_INVALID_ARGUMENT
