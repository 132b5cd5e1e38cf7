"""CPU oracle for the ConvRot quantized-linear path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s
CPU-baseline leg may import this module.  The shipped library never calls it and
has no CPU fallback.

The arithmetic lives in ``convrot_oracle.c`` (a plain-C restatement of the
reference kernels, see its header for the file:line it follows); this wrapper
compiles/loads it and adds the exact int32 contraction and int4 packing helpers.

Reference anchors (comfyui-turing-utils, kernel package 0.31.0):
  * rotate + quantize: ``kernel/csrc/turing/convrot_quant.cu:104-135,378-510``
  * int32 contraction: exact, pinned by ``kernel/scripts/validate_compatible.py:124-136``
  * epilogue: ``kernel/csrc/turing/w4a8.cu:474-525``, ``bf16_epilogue.cu:105-113``
  * signed int4 packing: ``kernel/csrc/turing/w4a8.cu:34-72``,
    ``kernel/scripts/validate_compatible.py:28-40``
  * RMSNorm / LayerNorm + AdaLN: ``kernel/csrc/turing/segmented_rms_adaln.cu:75-297``
    (exact reduction order; the device rsqrtf is replaced by a correctly rounded
    1/sqrt, so results may differ from the device by one output ulp)
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "convrot_oracle.c"
_LIB_PATH = _HERE / "libconvrot_oracle.so"
_lib = None

MODE_PLAIN = 0
MODE_SWIGLU = 1
MODE_GELU = 2
MODE_GELU_UNCONTRACTED = 3


def build(force: bool = False) -> Path:
    """Compile the C restatement (gcc, IEEE float, no contraction)."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < _SRC.stat().st_mtime:
        tmp = _LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(
            [
                "gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
                "-fPIC", "-shared", "-o", str(tmp), str(_SRC), "-lm",
            ],
            check=True,
        )
        os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_long, ctypes.c_int
        lib.ctu_oracle_convrot_quantize.argtypes = [vp, vp, vp, i64, i32, i32, i32]
        lib.ctu_oracle_convrot_quantize.restype = i32
        lib.ctu_oracle_convrot_quantize_staged.argtypes = [vp, vp, vp, i64, i32, i32, i32]
        lib.ctu_oracle_convrot_quantize_staged.restype = i32
        lib.ctu_oracle_convrot_quantize_staged_f16.argtypes = [vp, vp, vp, i64, i32, i32, i32]
        lib.ctu_oracle_convrot_quantize_staged_f16.restype = i32
        lib.ctu_oracle_convrot_quantize_scaled_f16.argtypes = [vp, vp, vp, i64, i32]
        lib.ctu_oracle_convrot_quantize_scaled_f16.restype = i32
        lib.ctu_oracle_convrot_quantize_scaled.argtypes = [vp, vp, vp, i64, i32, i32]
        lib.ctu_oracle_convrot_quantize_scaled.restype = i32
        lib.ctu_oracle_set_threads.argtypes = [i32]
        lib.ctu_oracle_set_threads.restype = None
        lib.ctu_oracle_get_threads.argtypes = []
        lib.ctu_oracle_get_threads.restype = i32
        lib.ctu_oracle_codebook_decode.argtypes = [vp, vp, vp, vp, i64, i32, i32]
        lib.ctu_oracle_codebook_decode.restype = None
        lib.ctu_oracle_rotate.argtypes = [vp, vp, i64, i32, i32]
        lib.ctu_oracle_rotate.restype = None
        lib.ctu_oracle_epilogue.argtypes = [vp, i64, vp, vp, i64, vp, vp, i64, i64, i32, i32]
        lib.ctu_oracle_epilogue.restype = None
        lib.ctu_oracle_segmented_rms_adaln.argtypes = [vp, vp, vp, vp, vp, vp, i64, i32, i32, i64, i64, i32,
                                                       ctypes.c_float, i32, i32]
        lib.ctu_oracle_segmented_rms_adaln.restype = None
        lib.ctu_oracle_layer_norm_adaln.argtypes = [vp, vp, vp, vp, i64, i64, i32, i32, ctypes.c_float, i32]
        lib.ctu_oracle_layer_norm_adaln.restype = None
        lib.ctu_oracle_convrot_quantize_int4_g128.argtypes = [vp, vp, vp, i64, i32]
        lib.ctu_oracle_convrot_quantize_int4_g128.restype = i32
        lib.ctu_oracle_grouped_epilogue.argtypes = [vp, i32, vp, vp, vp, vp, i64, i64, i32]
        lib.ctu_oracle_grouped_epilogue.restype = None
        lib.ctu_oracle_convrot_quantize_int4_g128_b128.argtypes = [vp, vp, vp, i64, i32]
        lib.ctu_oracle_convrot_quantize_int4_g128_b128.restype = i32
        lib.ctu_oracle_convrot_quantize_b128.argtypes = [vp, vp, vp, i64, i32]
        lib.ctu_oracle_convrot_quantize_b128.restype = i32
        lib.ctu_oracle_rotate_group_b128.argtypes = [vp, vp]
        lib.ctu_oracle_rotate_group_b128.restype = None
        lib.ctu_oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.ctu_oracle_f32_to_bf16.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def set_threads(threads: int) -> int:
    """OpenMP worker threads of the C restatement; returns the count now in effect."""
    lib = _load()
    lib.ctu_oracle_set_threads(int(threads))
    return lib.ctu_oracle_get_threads()


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (RNE, NaN -> 0x7fff) and return the uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    upper = (bits >> 16).astype(np.uint32)
    rem = bits & 0xFFFF
    round_up = (rem > 0x8000) | ((rem == 0x8000) & ((upper & 1) == 1))
    out = (upper + round_up).astype(np.uint16)
    nan = (bits & 0x7FFFFFFF) > 0x7F800000
    out[nan] = 0x7FFF
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rotate(x_bits: np.ndarray, mode: int = MODE_PLAIN) -> np.ndarray:
    """fp32 rotated activations (before bf16 rounding) for a [M, K] (or [M, 2K]) bf16 row block."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, width = x_bits.shape
    k = width // 2 if mode == MODE_SWIGLU else width
    y = np.empty((rows, k), dtype=np.float32)
    _load().ctu_oracle_rotate(_ptr(x_bits), _ptr(y), rows, k, mode)
    return y


def convrot_quantize(x_bits: np.ndarray, bits: int = 8, mode: int = MODE_PLAIN, staged: bool = False):
    """Reference ConvRot row quantizer on bf16 bit patterns.

    Returns ``(codes, scales)``: int8 ``[M, K]`` (bits=8) or packed int4 ``[M, K/2]``
    (bits=4), and fp32 ``[M]`` per-token scales.  ``staged`` selects the scale formula
    of the reference's staged quantizers (absmax times the fp32 reciprocal of qmax,
    convrot_quant.cu:300-303,335-338) instead of the row-buffer kernel's division.
    """
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, width = x_bits.shape
    k = width // 2 if mode == MODE_SWIGLU else width
    if k % 256 != 0:
        raise ValueError("ConvRot requires K divisible by 256")
    codes = np.empty((rows, k // 2 if bits == 4 else k), dtype=np.int8)
    scales = np.empty((rows,), dtype=np.float32)
    fn = _load().ctu_oracle_convrot_quantize_staged if staged else _load().ctu_oracle_convrot_quantize
    rc = fn(_ptr(x_bits), _ptr(codes), _ptr(scales), rows, k, bits, mode)
    if rc != 0:
        raise ValueError(f"unsupported ConvRot width {k}")
    return codes, scales


def convrot_quantize_staged_f16(x_bits: np.ndarray, bits: int = 8, mode: int = MODE_SWIGLU):
    """The staged SwiGLU / GELU quantizers on fp16 bit patterns (convrot_quant.cu:184-358
    with InputType = half): ``(codes, scales)`` like convrot_quantize."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, width = x_bits.shape
    k = width // 2 if mode == MODE_SWIGLU else width
    codes = np.empty((rows, k // 2 if bits == 4 else k), dtype=np.int8)
    scales = np.empty((rows,), dtype=np.float32)
    rc = _load().ctu_oracle_convrot_quantize_staged_f16(_ptr(x_bits), _ptr(codes), _ptr(scales), rows, k, bits,
                                                        1 if mode == MODE_SWIGLU else 2)
    if rc != 0:
        raise ValueError(f"unsupported ConvRot width {k} or mode {mode}")
    return codes, scales


def convrot_quantize_scaled_f16(x_bits: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """turing_swiglu_int8_convrot_quantize_scaled on fp16 bit patterns."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, width = x_bits.shape
    k = width // 2
    scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
    codes = np.empty((rows, k), dtype=np.int8)
    if _load().ctu_oracle_convrot_quantize_scaled_f16(_ptr(x_bits), _ptr(scales), _ptr(codes), rows, k) != 0:
        raise ValueError(f"unsupported ConvRot width {k}")
    return codes


def convrot_quantize_scaled(x_bits: np.ndarray, scales: np.ndarray, mode: int = MODE_SWIGLU) -> np.ndarray:
    """int8 codes of the rotated rows with caller-supplied per-row scales
    (``turing_swiglu_int8_convrot_quantize_scaled``, convrot_quant.cu:138-161,239-278)."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, width = x_bits.shape
    k = width // 2 if mode == MODE_SWIGLU else width
    scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
    codes = np.empty((rows, k), dtype=np.int8)
    rc = _load().ctu_oracle_convrot_quantize_scaled(_ptr(x_bits), _ptr(scales), _ptr(codes), rows, k, mode)
    if rc != 0:
        raise ValueError(f"unsupported ConvRot width {k}")
    return codes


def int8_gemm_s32(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Exact int32 contraction ``a[M,K] @ w[N,K]^T`` (no overflow for K < 131072)."""
    import torch

    a_t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int8))
    w_t = torch.from_numpy(np.ascontiguousarray(w, dtype=np.int8))
    m, k = a_t.shape
    n = w_t.shape[0]
    if m >= 17 and n % 8 == 0 and k % 8 == 0:
        return torch._int_mm(a_t, w_t.t().contiguous()).numpy()
    return (a_t.to(torch.int64) @ w_t.to(torch.int64).t()).to(torch.int32).numpy()


def epilogue(acc: np.ndarray, a_scale: np.ndarray, w_scale: np.ndarray, bias=None,
             fused: bool = True, add_zero_bias: bool = True) -> np.ndarray:
    """bf16 bits of ``fma(acc * a_s, w_s, bias)`` (w4a8.cu:474-525).

    The reference's GEMM epilogue is compiled with nvcc's default FMA contraction, which
    fuses the weight-scale multiply and the bias add (``fused=True``, the default; its
    outputs match this on every element of a 32760 x 5120 x 5120 linear run on B200).
    ``fused=False`` rounds the product and the sum separately.

    ``bias=None`` with ``add_zero_bias`` mirrors the GEMM's null bias broadcast (a
    +0.0 addition); ``add_zero_bias=False`` mirrors ``turing_dequantize_int8_bf16``
    (bf16_epilogue.cu:105-113), which has no addition.
    """
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    m, n = acc.shape
    a_scale = np.ascontiguousarray(a_scale, dtype=np.float32).reshape(-1)
    w_scale = np.ascontiguousarray(w_scale, dtype=np.float32).reshape(-1)
    has_bias = 1
    if bias is None:
        if add_zero_bias:
            bias = np.zeros((n,), dtype=np.float32)
        else:
            has_bias = 0
            bias = np.zeros((1,), dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    out = np.empty((m, n), dtype=np.uint16)
    _load().ctu_oracle_epilogue(
        _ptr(acc), n, _ptr(a_scale), _ptr(w_scale), w_scale.size, _ptr(bias), _ptr(out),
        m, n, has_bias, 1 if fused else 0,
    )
    return out


def pack_int4(values: np.ndarray) -> np.ndarray:
    """Signed int4 values in [-8, 7] -> packed bytes, even column in the low nibble."""
    v = np.asarray(values, dtype=np.int32)
    lo = v[:, 0::2] & 0x0F
    hi = v[:, 1::2] & 0x0F
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Packed bytes -> signed int4 values as int8, low nibble first (w4a8.cu:49-66)."""
    p = np.asarray(packed).view(np.uint8).astype(np.int32)
    lo = p & 0x0F
    hi = (p >> 4) & 0x0F
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.stack((lo, hi), axis=-1).reshape(p.shape[0], -1)
    return out.astype(np.int8)


def int8_linear(a, w, a_scale, w_scale, bias=None, fused=True):
    """``turing_utils::int8_linear`` oracle: bf16 bits [M, N]."""
    return epilogue(int8_gemm_s32(a, w), a_scale, w_scale, bias, fused=fused)


def w4a8_linear(a, w_packed, a_scale, w_scale, bias=None, fused=True):
    """``turing_utils::w4a8_linear`` oracle (signed int4 weights, per-channel scale)."""
    return epilogue(int8_gemm_s32(a, unpack_int4(w_packed)), a_scale, w_scale, bias, fused=fused)


def w4a4_linear(a_packed, w_packed, a_scale, w_scale, bias=None, fused=True):
    """W4A4: packed signed-int4 activation codes x packed signed-int4 weights, the same
    epilogue.  The reference's int4 GEMM is comfy-kitchen's (source not available), so
    this definition -- exact int32 contraction of the sign-extended values, then the
    bundled kernels' epilogue -- is this build's, not a restatement (parity unpinned)."""
    return epilogue(int8_gemm_s32(unpack_int4(a_packed), unpack_int4(w_packed)), a_scale, w_scale, bias, fused=fused)


def convrot_w8a8_linear(x_bits, w, w_scale, bias=None, fused=True):
    """Whole path: ConvRot quantize, int32 GEMM, dequant+bias epilogue (bf16 bits)."""
    codes, scales = convrot_quantize(x_bits, 8)
    return int8_linear(codes, w, scales, w_scale, bias, fused=fused)


def codebook_decode(w_packed: np.ndarray, group_scale: np.ndarray, codebook: np.ndarray, group_size: int) -> np.ndarray:
    """Grouped-codebook W4 weights -> int8 [N, K] (w4a8.cu:903-976): e4m3fn group scale
    (raw bytes [N, K/group_size]) times a 16-entry fp32 codebook, rint, clamp +-127."""
    w_packed = np.ascontiguousarray(w_packed).view(np.int8)
    rows, half = w_packed.shape
    k = 2 * half
    group_scale = np.ascontiguousarray(group_scale).view(np.uint8)
    codebook = np.ascontiguousarray(codebook, dtype=np.float32).reshape(-1)
    if codebook.size != 16 or group_scale.shape != (rows, k // group_size):
        raise ValueError("codebook must have 16 entries and group_scale shape [N, K/group_size]")
    out = np.empty((rows, k), dtype=np.int8)
    _load().ctu_oracle_codebook_decode(_ptr(w_packed), _ptr(group_scale), _ptr(codebook), _ptr(out), rows, k,
                                       group_size)
    return out


def codebook_w4a8_linear(a, w_packed, a_scale, group_scale, channel_scale, codebook, bias=None, group_size=16):
    """``turing_utils::codebook_w4a8_linear`` oracle: decode, exact int32 GEMM, then the
    W8A8 epilogue with the per-channel scale (w4a8.cu:1088-1182)."""
    w = codebook_decode(w_packed, group_scale, codebook, group_size)
    return int8_linear(a, w, a_scale, channel_scale, bias)


# ---------------------------------------------------------------------------------------
# Per-group-128 formats (configs of the W4A8 / W4A4 linears).  The reference runs these
# through comfy-kitchen (dispatch.py:876-936), whose source is not available: the
# definitions here are this build's (parity unpinned), see convrot_oracle.c.
QGROUP = 128


def convrot_quantize_int4_g128(x_bits: np.ndarray, block: int = 256):
    """Rotate (block 256: the reference's rotation; 128: this build's block-128 rotation),
    then per-token-per-group-128 int4: ``(codes [M, K/2] packed, scales [M, K/128])``."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, k = x_bits.shape
    codes = np.empty((rows, k // 2), dtype=np.int8)
    scales = np.empty((rows, max(k // QGROUP, 1)), dtype=np.float32)
    fn = (_load().ctu_oracle_convrot_quantize_int4_g128_b128 if block == 128
          else _load().ctu_oracle_convrot_quantize_int4_g128)
    if fn(_ptr(x_bits), _ptr(codes), _ptr(scales), rows, k) != 0:
        raise ValueError(f"unsupported ConvRot width {k}")
    return codes, scales


RSQRT2_F32 = np.float32(0.70710676908493042)  # RN_fp32(1 / sqrt 2) = 0x1.6a09e6p-1


def convrot_quantize_b128(x_bits: np.ndarray):
    """Rotation block 128 (this build's definition, parity unpinned: the reference's ops
    take 256 only): the reference's radix-4 stages at strides 1, 4, 16, then a radix-2
    stage at stride 64, ``y0 = (x0 + x1) * c, y1 = (x0 - x1) * c`` with c = RN(1/sqrt 2),
    then the int8 chain of the 256 rotation.  Returns ``(codes [M, K] int8, scales [M])``."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, k = x_bits.shape
    codes = np.empty((rows, k), dtype=np.int8)
    scales = np.empty((rows,), dtype=np.float32)
    if _load().ctu_oracle_convrot_quantize_b128(_ptr(x_bits), _ptr(codes), _ptr(scales), rows, k) != 0:
        raise ValueError(f"unsupported ConvRot width {k}")
    return codes, scales


def rotate_group_b128(values: np.ndarray) -> np.ndarray:
    """The fp32 block-128 rotation of one 256-column group (two independent 128-blocks)."""
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(256)
    out = np.empty(256, dtype=np.float32)
    _load().ctu_oracle_rotate_group_b128(_ptr(v), _ptr(out))
    return out


def widen_uint4_zero(w_packed: np.ndarray, zeros: np.ndarray) -> np.ndarray:
    """Asymmetric uint4 weights [N, K/2] (even column in the low nibble) and uint4 zero
    points [N, K/128] -> the int8 values ``nibble - zero`` [N, K] in [-15, 15]."""
    p = np.asarray(w_packed).view(np.uint8).astype(np.int16)
    n = p.shape[0]
    vals = np.stack((p & 0x0F, (p >> 4) & 0x0F), axis=-1).reshape(n, -1)
    z = np.repeat(np.asarray(zeros, dtype=np.uint8).astype(np.int16), QGROUP, axis=1)
    return (vals - z).astype(np.int8)


def grouped_partials(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Exact int32 partial products of every 128-column group: [K/128, M, N]."""
    k = a.shape[1]
    return np.stack([int8_gemm_s32(a[:, g:g + QGROUP], w[:, g:g + QGROUP]) for g in range(0, k, QGROUP)])


def grouped_epilogue(partials: np.ndarray, a_scale: np.ndarray, w_scale_gn: np.ndarray, bias, mode: int) -> np.ndarray:
    """bf16 bits of the per-group epilogue (mode 0: W4A8 per-token activation scale;
    mode 1: W4A4 per-token-per-group activation scale), see convrot_oracle.c."""
    partials = np.ascontiguousarray(partials, dtype=np.int32)
    groups, m, n = partials.shape
    a_scale = np.ascontiguousarray(a_scale, dtype=np.float32)
    w_scale_gn = np.ascontiguousarray(w_scale_gn, dtype=np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    out = np.empty((m, n), dtype=np.uint16)
    _load().ctu_oracle_grouped_epilogue(_ptr(partials), groups, _ptr(a_scale), _ptr(w_scale_gn),
                                        None if bias_arr is None else _ptr(bias_arr), _ptr(out), m, n, mode)
    return out


def _group_major(w_scale) -> np.ndarray:
    """fp16 checkpoint scales [N, K/128] -> fp32 [K/128, N]."""
    return np.ascontiguousarray(np.asarray(w_scale, dtype=np.float16).astype(np.float32).T)


def asym_w4a8_g128_linear(a, w_packed, a_scale, w_scale, w_zero, bias=None):
    """Asymmetric uint4 W4A8 with fp16 scale and uint4 zero point per 128 columns:
    a int8 [M, K], a_scale [M], w_packed uint8 [N, K/2], w_scale fp16 [N, K/128],
    w_zero uint8 [N, K/128] -> bf16 bits [M, N]."""
    w = widen_uint4_zero(w_packed, w_zero)
    return grouped_epilogue(grouped_partials(a, w), np.asarray(a_scale).reshape(-1), _group_major(w_scale), bias, 0)


def w4a4_g128_linear(a_packed, w_packed, a_scale, w_scale, bias=None):
    """Symmetric int4 x int4 with per-token-per-group activation scales a_scale [M, K/128]
    and fp16 weight scales w_scale [N, K/128] -> bf16 bits [M, N]."""
    a = unpack_int4(a_packed)
    w = unpack_int4(w_packed)
    return grouped_epilogue(grouped_partials(a, w), a_scale, _group_major(w_scale), bias, 1)

# Storage-type codes of the norm ops (bf16 and fp16 travel as uint16 bit patterns).
NORM_BF16, NORM_FP16, NORM_FP32 = 0, 1, 2


def _norm_array(a: np.ndarray, dtype: int) -> np.ndarray:
    want = np.float32 if dtype == NORM_FP32 else np.uint16
    if a.dtype != want:
        raise TypeError(f"norm oracle expects {want.__name__} storage for dtype code {dtype}")
    return np.ascontiguousarray(a)


def segmented_rms_adaln(x, weight, scale, shift, segments, epsilon: float, dtype: int, vectorized: bool,
                        scale_stride: int | None = None, shift_stride: int | None = None,
                        param_rows: int | None = None) -> np.ndarray:
    """segmented_rms_adaln.cu:133-232.  x [rows, hidden]; weight [hidden]; scale/shift
    [param_rows, stride] (rows `*_stride` elements apart, first `hidden` used);
    segments int32 [S, 3].  ``vectorized`` is the reference launch's choice (:308-313)."""
    x, weight = _norm_array(x, dtype), _norm_array(weight, dtype)
    scale, shift = _norm_array(scale, dtype), _norm_array(shift, dtype)
    segments = np.ascontiguousarray(segments, dtype=np.int32)
    rows, hidden = x.shape
    out = np.empty_like(x)
    _load().ctu_oracle_segmented_rms_adaln(
        _ptr(x), _ptr(weight), _ptr(scale), _ptr(shift), _ptr(segments), _ptr(out), rows, hidden,
        param_rows if param_rows is not None else scale.shape[0],
        scale_stride if scale_stride is not None else scale.shape[1],
        shift_stride if shift_stride is not None else shift.shape[1], segments.shape[0], float(epsilon), dtype,
        1 if vectorized else 0)
    return out


def layer_norm_adaln(x, scale, shift, epsilon: float, dtype: int) -> np.ndarray:
    """segmented_rms_adaln.cu:234-297.  x [batch, sequence, hidden]; scale/shift
    [batch, modulation_steps, hidden]."""
    x, scale, shift = _norm_array(x, dtype), _norm_array(scale, dtype), _norm_array(shift, dtype)
    batch, sequence, hidden = x.shape
    out = np.empty_like(x)
    _load().ctu_oracle_layer_norm_adaln(_ptr(x), _ptr(scale), _ptr(shift), _ptr(out), batch, sequence, hidden,
                                        scale.shape[1], float(epsilon), dtype)
    return out

