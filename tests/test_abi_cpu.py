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


def test_c99_binding_links_and_reports_errors(tmp_path):
    """include/ctu_b200.h compiles as strict C99 and the built library links into a C
    program (as a cgo / N-API / JNI binding would use it); tests/native/abi_c99.c checks
    the argument contracts, sizes and host-side plans there, without a GPU."""
    import shutil
    import subprocess

    from comfyui_turing_utils_kernel import _lib

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lib_path = _lib.library_path()
    exe = tmp_path / "abi_c99"
    subprocess.run(["gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    "-o", str(exe), str(ROOT / "tests" / "native" / "abi_c99.c"), str(lib_path),
                    f"-Wl,-rpath,{lib_path.parent}"], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    assert "C99 ABI checks passed" in run.stdout


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


def test_fused_linear_contract_without_a_gpu():
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    # One claim counter plus one finished-row counter per 128-row block.
    assert [lib.ctu_convrot_int8_linear_sync_words(m) for m in (0, 1, 128, 129, 32760)] == [1, 2, 2, 3, 257]
    rc = lib.ctu_convrot_int8_linear(null, null, null, 8, null, null, null, null, null, 4, 8, 300, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "divisible by 256" in lib.ctu_last_error().decode()
    fake = ctypes.c_void_p(0x10000)  # aligned, never dereferenced: the shape check fails first
    rc = lib.ctu_convrot_int8_linear(fake, fake, fake, 12, null, fake, fake, fake, fake, 4, 12, 512, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "N%8=0" in lib.ctu_last_error().decode()
    rc = lib.ctu_convrot_int8_linear(null, null, null, 8, null, null, null, null, null, 0, 8, 512, null)
    assert rc == _lib.CTU_OK  # no rows: nothing to do
    assert lib.ctu_debug_set_fused_linear(3) == _lib.CTU_ERR_INVALID_ARGUMENT


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
    # host for B200's 227 KB of opt-in shared memory: the warp-row kernel for plain and GELU
    # rows of 4096 < K <= 6144 (four warps, one row each), the multi-group eight-lane kernel
    # for wider plain and GELU rows (two groups per team at K = 13824), eight lanes for
    # SwiGLU at K = 5120, four lanes at K <= 4096, and the two-pass kernel beyond K = 32768.
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    two_pass, reg, t4, k8, g8, w8 = 0, 1, 2, 3, 4, 5

    def plan(k, act=0, bits=8):
        kind, warps, rows = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        rc = lib.ctu_debug_quant_plan(k, act, bits, 232448, ctypes.byref(kind), ctypes.byref(warps), ctypes.byref(rows))
        assert rc == 0, lib.ctu_last_error().decode()
        return kind.value, warps.value, rows.value

    assert plan(5120) == (w8, 4, 4)
    assert plan(5120, act=2)[0] == w8 and plan(5120, bits=4)[0] == w8
    assert plan(6400)[0] == g8
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
        lib.ctu_debug_set_quant_kernel(7)
        assert plan(5120) == (g8, 5, 2)
        lib.ctu_debug_set_quant_kernel(8)
        assert plan(3072)[0] == w8 and plan(13824)[0] != w8  # wider than the warp-row kernel takes
    finally:
        lib.ctu_debug_set_quant_kernel(prev)
    assert lib.ctu_debug_quant_plan(300, 0, 8, 232448, ctypes.byref(ctypes.c_int()), ctypes.byref(ctypes.c_int()),
                                    ctypes.byref(ctypes.c_int())) == _lib.CTU_ERR_INVALID_ARGUMENT


def test_grouped_entry_points_reject_bad_shapes_without_a_gpu():
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    rc = lib.ctu_asym_w4a8_g128_linear(null, null, null, null, null, null, null, null, 4, 8, 192, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "K%128=0" in lib.ctu_last_error().decode()
    rc = lib.ctu_w4a4_g128_linear(null, null, null, null, null, null, null, null, 4, 12, 256, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "N%8=0" in lib.ctu_last_error().decode()
    rc = lib.ctu_convrot_quantize_int4_g128(null, 4, 384, null, null, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "divisible by 256" in lib.ctu_last_error().decode()
    assert lib.ctu_w4a4_g128_linear(null, null, null, null, null, null, null, null, 0, 16, 256, null) == _lib.CTU_OK
    assert lib.ctu_convrot_quantize_int4_g128(null, 0, 512, null, null, null) == _lib.CTU_OK


def test_grouped_custom_op_fake_shapes():
    import comfyui_turing_utils_kernel as k

    x = torch.empty((3, 512), dtype=torch.bfloat16, device="meta")
    q, s = k.turing_bf16_int4_g128_convrot_quantize(x, 256)
    assert q.shape == (3, 256) and q.dtype == torch.int8 and s.shape == (3, 4) and s.dtype == torch.float32
    a = torch.empty((7, 256), dtype=torch.int8, device="meta")
    w = torch.empty((16, 128), dtype=torch.uint8, device="meta")
    out = k.turing_asym_w4a8_g128_linear(a, w, torch.empty(7, device="meta"), torch.empty((16, 2), device="meta"),
                                         torch.empty((16, 2), dtype=torch.uint8, device="meta"))
    assert out.shape == (7, 16) and out.dtype == torch.bfloat16
    out = k.turing_w4a4_g128_linear(a[:, :128], w.view(torch.int8), torch.empty((7, 2), device="meta"),
                                    torch.empty((16, 2), device="meta"))
    assert out.shape == (7, 16)


def test_oracle_grouped_formats_against_float64():
    # The per-group oracle definitions reproduce the float64 dequantized product to the
    # accuracy of their fp32 accumulation and bf16 output.
    import numpy as np

    import convrot_oracle as oracle

    rng = np.random.default_rng(0)
    m, k, n = 37, 512, 48
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[:, rng.permutation(k)[:5]] *= 30
    xb = oracle.f32_to_bf16_bits(x)
    codes, scales = oracle.convrot_quantize_int4_g128(xb)
    assert codes.shape == (m, k // 2) and scales.shape == (m, k // 128)
    y = oracle.rotate(xb).astype(np.float64)
    deq = oracle.unpack_int4(codes).astype(np.float64) * np.repeat(scales.astype(np.float64), 128, axis=1)
    # int4 rounding: at most half a step of each group's scale (plus bf16 rounding of y).
    assert np.all(np.abs(deq - y) <= np.repeat(scales, 128, axis=1) * 0.5 * (1 + 2 ** -7) + np.abs(y) * 2 ** -8)

    wp = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    wz = rng.integers(0, 16, (n, k // 128), dtype=np.uint8)
    ws = (rng.random((n, k // 128)) * 0.009 + 1e-3).astype(np.float16)
    b = (rng.standard_normal(n) * 0.02).astype(np.float32)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    asc = (rng.random(m) * 0.01 + 1e-3).astype(np.float32)
    out = oracle.bf16_bits_to_f32(oracle.asym_w4a8_g128_linear(a, wp, asc, ws, wz, b)).astype(np.float64)
    w = oracle.widen_uint4_zero(wp, wz).astype(np.float64) * np.repeat(ws.astype(np.float64), 128, axis=1)
    ref = (a.astype(np.float64) @ w.T) * asc[:, None] + b
    assert np.max(np.abs(out - ref) / (np.abs(ref) + 1e-3)) < 2 ** -7

    w4 = rng.integers(-7, 8, (n, k)).astype(np.int8)
    out = oracle.bf16_bits_to_f32(oracle.w4a4_g128_linear(codes, oracle.pack_int4(w4), scales, ws, b))
    a_deq = oracle.unpack_int4(codes).astype(np.float64) * np.repeat(scales.astype(np.float64), 128, axis=1)
    w_deq = w4.astype(np.float64) * np.repeat(ws.astype(np.float64), 128, axis=1)
    ref = a_deq @ w_deq.T + b
    assert np.max(np.abs(out.astype(np.float64) - ref) / (np.abs(ref) + 1e-2)) < 2 ** -7


def test_block128_oracle_is_the_kronecker_rotation():
    # The block-128 rotation of the oracle is (1/sqrt 2) H2 (x) M (x) M (x) M on each 128-column
    # block (M the reference's radix-4 stage): compare it with that matrix in float64.
    import numpy as np

    import convrot_oracle as oracle

    m4 = 0.5 * np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
    h2 = np.array([[1, 1], [1, -1]], dtype=np.float64) / np.sqrt(2.0)
    t = np.kron(h2, np.kron(m4, np.kron(m4, m4)))
    assert np.allclose(t @ t.T, np.eye(128), atol=1e-12)  # orthogonal
    rng = np.random.default_rng(5)
    for _ in range(20):
        x = (rng.standard_normal(256) * rng.choice([1e-3, 1.0, 30.0], 256)).astype(np.float32)
        y = oracle.rotate_group_b128(x).astype(np.float64)
        ref = np.concatenate([t @ x[:128].astype(np.float64), t @ x[128:].astype(np.float64)])
        assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


def test_block128_entry_rejects_bad_widths_without_a_gpu():
    import ctypes

    from comfyui_turing_utils_kernel import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    rc = lib.ctu_convrot_quantize_b128(null, 4, 384, null, null, null)
    assert rc == _lib.CTU_ERR_INVALID_ARGUMENT and "divisible by 256" in lib.ctu_last_error().decode()
    assert lib.ctu_convrot_quantize_b128(null, 0, 512, null, null, null) == _lib.CTU_OK
