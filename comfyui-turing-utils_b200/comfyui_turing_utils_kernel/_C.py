"""Drop-in for the reference's native module ``comfyui_turing_utils_kernel._C``.

Same attribute names, argument names, defaults, output allocation and error
contract as the reference's pybind11 bindings (kernel/csrc/bindings.cpp:884-973),
implemented over the C ABI of libctu_b200.so.  Torch is used only for device
memory, the current stream and the device guard.

Attributes that the reference exposes but this build does not implement are
absent, so ``hasattr(_C, name)`` probes (kernel_api.py:26-37, dispatch.py:59-69)
stay truthful.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_lib.load()  # fail at import time when the CUDA library is missing (no fallback)


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check_cuda_2d(t: torch.Tensor, name: str) -> None:
    # bindings.cpp:89-93
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dim() != 2:
        raise RuntimeError(f"{name} must be 2D")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The C ABI wants 16-byte aligned rows; copy the rare misaligned view."""
    if t.data_ptr() % 16 == 0:
        return t
    out = torch.empty_like(t, memory_format=torch.contiguous_format)
    out.copy_(t)
    return out


# ----------------------------------------------------------------------------- quantizers
def _convrot_quantize(x: torch.Tensor, group_size: int, act: int, bits: int, what: str, staged: bool = False):
    x = x.contiguous()
    _check_cuda_2d(x, "input")
    if staged:  # the staged quantizers take fp16 rows too (check_half_like, bindings.cpp:95-99)
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise RuntimeError("input must be float16 or bfloat16")
    elif x.dtype != torch.bfloat16:
        raise RuntimeError(f"{what} input must be bfloat16")
    if group_size != 256:
        raise RuntimeError(f"{what} only supports group_size=256")
    rows, width = x.shape
    if act == _lib.ACT_SWIGLU and width % 2 != 0:
        raise RuntimeError(f"SwiGLU {what} input width must be even")
    hidden = width // 2 if act == _lib.ACT_SWIGLU else width
    if rows <= 0 or hidden <= 0 or hidden % group_size != 0:
        raise RuntimeError(f"{what} width must be positive and divisible by 256")
    x = _aligned(x)
    codes = torch.empty((rows, hidden // 2 if bits == 4 else hidden), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        if staged:
            _lib.check(_lib.load().ctu_convrot_quantize_staged(
                _ptr(x), rows, hidden, act, bits, _NORM_TYPES[x.dtype], _ptr(codes), _ptr(scales), _stream(x.device)))
        else:
            _lib.check(_lib.load().ctu_convrot_quantize(
                _ptr(x), rows, hidden, act, bits, _ptr(codes), _ptr(scales), _stream(x.device)))
    return codes, scales


def turing_bf16_int8_convrot_quantize(input, group_size=256, swiglu=False, forced_threads=0):
    """bindings.cpp:636-679.  ``forced_threads`` selected the SM75 block geometry; the
    B200 kernel's geometry is fixed, so only the reference's value check remains."""
    if forced_threads not in (0, 512, 768, 1024):
        raise RuntimeError("forced_threads must be 0, 512, 768, or 1024")
    act = _lib.ACT_SWIGLU if swiglu else _lib.ACT_NONE
    return _convrot_quantize(input, group_size, act, 8, "BF16 row-buffer ConvRot")


def bf16_int8_convrot_quantize_b128(input):
    """ConvRot int8 quantize with rotation block 128 (this library's definition, parity
    unpinned: the reference's ops take 256 only; see ctu_b200.h).  Returns the int8
    codes [M, K] and the per-token scales [M, 1]."""
    x = input.contiguous()
    _check_cuda_2d(x, "input")
    if x.dtype != torch.bfloat16:
        raise RuntimeError("block-128 ConvRot input must be bfloat16")
    rows, width = x.shape
    if rows <= 0 or width <= 0 or width % 256 != 0:
        raise RuntimeError("block-128 ConvRot width must be positive and divisible by 256")
    x = _aligned(x)
    codes = torch.empty((rows, width), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().ctu_convrot_quantize_b128(_ptr(x), rows, width, _ptr(codes), _ptr(scales),
                                                         _stream(x.device)))
    return codes, scales


def turing_bf16_int4_convrot_quantize(input, group_size=256, swiglu=False):
    """bindings.cpp:681-717."""
    act = _lib.ACT_SWIGLU if swiglu else _lib.ACT_NONE
    return _convrot_quantize(input, group_size, act, 4, "BF16 row-buffer INT4 ConvRot")


def turing_bf16_gelu_int8_convrot_quantize(input, group_size=256):
    """bindings.cpp:719-770 (int8)."""
    return _convrot_quantize(input, group_size, _lib.ACT_GELU_TANH, 8, "BF16 GELU row-buffer ConvRot")


def turing_bf16_gelu_int4_convrot_quantize(input, group_size=256):
    """bindings.cpp:719-770 (int4)."""
    return _convrot_quantize(input, group_size, _lib.ACT_GELU_TANH, 4, "BF16 GELU row-buffer ConvRot")


# The reference's staged two-kernel quantizers (convrot_quant.cu:184-358) rotate and
# round exactly like the row-buffer kernel but form the row scale as absmax * (1/qmax)
# instead of absmax / qmax (their own validation compares the two scales with rtol 1e-6,
# validate_compatible.py:43-64).  On B200 both names run the same fused kernels, the
# staged names with the staged scale, so each matches its reference op bit for bit.
# Like the reference, the staged entries also take fp16 rows (rounded to fp16 where the
# bf16 path rounds to bf16; the two-pass kernel runs them).
def turing_swiglu_int8_convrot_quantize(input, group_size=256):
    """bindings.cpp:474-510."""
    return _convrot_quantize(input, group_size, _lib.ACT_SWIGLU, 8, "SwiGLU staged ConvRot", staged=True)


def turing_swiglu_int4_convrot_quantize(input, group_size=256):
    """bindings.cpp:547-584."""
    return _convrot_quantize(input, group_size, _lib.ACT_SWIGLU, 4, "SwiGLU staged INT4 ConvRot", staged=True)


def turing_gelu_int8_convrot_quantize(input, group_size=256):
    """bindings.cpp:586-633 (int8)."""
    return _convrot_quantize(input, group_size, _lib.ACT_GELU_TANH, 8, "GELU staged ConvRot", staged=True)


def turing_gelu_int4_convrot_quantize(input, group_size=256):
    """bindings.cpp:586-633 (int4)."""
    return _convrot_quantize(input, group_size, _lib.ACT_GELU_TANH, 4, "GELU staged ConvRot", staged=True)


def turing_swiglu_int8_convrot_quantize_scaled(input, scales, group_size=256):
    """bindings.cpp:512-545: SwiGLU + ConvRot of one channel shard, int8 codes with the
    caller's whole-row scales (fp32, one per row); returns the codes only."""
    input = input.contiguous()
    scales = scales.reshape(-1).to(torch.float32).contiguous()
    _check_cuda_2d(input, "input")
    if input.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("input must be float16 or bfloat16")
    if group_size != 256:
        raise RuntimeError("scaled SwiGLU ConvRot only supports group_size=256")
    if input.shape[1] % 2 != 0:
        raise RuntimeError("scaled SwiGLU input width must be even")
    rows, hidden = input.shape[0], input.shape[1] // 2
    if rows <= 0 or hidden <= 0 or hidden % group_size != 0:
        raise RuntimeError("scaled SwiGLU width must be positive and divisible by 256")
    if not scales.is_cuda or scales.device != input.device or scales.numel() != rows:
        raise RuntimeError("scaled SwiGLU requires one FP32 scale per input row")
    input = _aligned(input)
    codes = torch.empty((rows, hidden), dtype=torch.int8, device=input.device)
    with torch.cuda.device(input.device):
        _lib.check(_lib.load().ctu_swiglu_int8_convrot_quantize_scaled(
            _ptr(input), rows, hidden, _NORM_TYPES[input.dtype], _ptr(scales), _ptr(codes), _stream(input.device)))
    return codes


# ----------------------------------------------------------------------------- GEMMs
def turing_int8_linear(activation, weight, activation_scale, weight_scale, bias=None, tile_policy=0):
    """bindings.cpp:371-421: W8A8 GEMM with the fused dequant + bias epilogue.
    ``tile_policy`` chose among SM75 CUTLASS tiles; the tcgen05 kernel has one
    persistent tile schedule, so the argument is accepted and ignored."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = activation_scale.reshape(-1).to(torch.float32).contiguous()
    weight_scale = weight_scale.reshape(-1).to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(torch.float32).contiguous()
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    if activation.dtype != torch.int8 or weight.dtype != torch.int8:
        raise RuntimeError("Turing INT8 linear activation and weight must be int8")
    dev = activation.device
    if weight.device != dev or activation_scale.device != dev or weight_scale.device != dev:
        raise RuntimeError("Turing INT8 linear tensors must use the same CUDA device")
    m, k = activation.shape
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise RuntimeError("INT8 linear K dimensions must match")
    if k % 16 != 0 or n % 8 != 0:
        raise RuntimeError("Turing INT8 linear requires K%16=0 and N%8=0")
    if activation_scale.numel() != m:
        raise RuntimeError("activation_scale must contain one value per row")
    if weight_scale.numel() != n:
        raise RuntimeError("weight_scale must contain one value per output channel")
    if bias is not None and (not bias.is_cuda or bias.device != dev or bias.numel() != n):
        raise RuntimeError("bias must contain one value per output channel on the same CUDA device")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    if m == 0 or n == 0 or k == 0:
        return out  # the reference leaves the output unwritten for empty problems (w4a8.cu:1194-1196)
    activation, weight = _aligned(activation), _aligned(weight)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ctu_int8_linear(
            _ptr(activation), _ptr(weight), _ptr(activation_scale), _ptr(weight_scale), n,
            _ptr(bias), _ptr(out), m, n, k, _stream(dev)))
    return out


def convrot_int8_linear(input, weight, weight_scale, bias=None, group_size=256, return_quantized=False):
    """ConvRot W8A8 linear from bf16 rows: the plugin's dispatch.int8_linear for plain rows
    (dispatch.py:748-800: turing_bf16_int8_convrot_quantize, then turing_int8_linear) as one
    library call.  Codes, scales and outputs equal those of the two ops bit for bit; for
    K <= 5120 one kernel quantizes rows while its tensor cores work on finished ones.
    ``return_quantized`` also returns the int8 codes [M, K] and scales [M, 1]."""
    x = input.contiguous()
    _check_cuda_2d(x, "input")
    if x.dtype != torch.bfloat16:
        raise RuntimeError("ConvRot INT8 linear input must be bfloat16")
    if group_size != 256:
        raise RuntimeError("ConvRot INT8 linear only supports group_size=256")
    weight = weight.contiguous()
    _check_cuda_2d(weight, "weight")
    if weight.dtype != torch.int8:
        raise RuntimeError("Turing INT8 linear activation and weight must be int8")
    weight_scale = weight_scale.reshape(-1).to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(torch.float32).contiguous()
    dev = x.device
    if weight.device != dev or weight_scale.device != dev:
        raise RuntimeError("Turing INT8 linear tensors must use the same CUDA device")
    m, k = x.shape
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise RuntimeError("INT8 linear K dimensions must match")
    if m <= 0 or k <= 0 or k % group_size != 0:
        raise RuntimeError("BF16 row-buffer ConvRot width must be positive and divisible by 256")
    if n % 8 != 0:
        raise RuntimeError("Turing INT8 linear requires K%16=0 and N%8=0")
    if weight_scale.numel() != n:
        raise RuntimeError("weight_scale must contain one value per output channel")
    if bias is not None and (not bias.is_cuda or bias.device != dev or bias.numel() != n):
        raise RuntimeError("bias must contain one value per output channel on the same CUDA device")
    lib = _lib.load()
    x, weight = _aligned(x), _aligned(weight)
    codes = torch.empty((m, k), dtype=torch.int8, device=dev)
    scales = torch.empty((m, 1), dtype=torch.float32, device=dev)
    sync = torch.empty((lib.ctu_convrot_int8_linear_sync_words(m),), dtype=torch.int32, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    if n > 0:
        with torch.cuda.device(dev):
            _lib.check(lib.ctu_convrot_int8_linear(
                _ptr(x), _ptr(weight), _ptr(weight_scale), n, _ptr(bias), _ptr(out), _ptr(codes), _ptr(scales),
                _ptr(sync), m, n, k, _stream(dev)))
    return (out, codes, scales) if return_quantized else out


# From this many activation rows on, the W4 linears widen their packed int4 operands to
# int8 once (a streaming pass) and run the W8A8 tensor-core GEMM, instead of widening every
# weight tile inside the GEMM for each row block: the pass costs about as much as the GEMM
# gains at ~500 rows of a 5120x5120 linear.
W4_WIDEN_MIN_ROWS = 512


def _widen_s4(packed: torch.Tensor) -> torch.Tensor:
    rows, half = packed.shape
    out = torch.empty((rows, 2 * half), dtype=torch.int8, device=packed.device)
    with torch.cuda.device(packed.device):
        _lib.check(_lib.load().ctu_int4_unpack_s8(_ptr(_aligned(packed)), _ptr(out), rows, 2 * half,
                                                  _stream(packed.device)))
    return out


def turing_w4a8_linear(activation, weight, activation_scale, weight_scale, bias=None, tile_policy=0):
    """bindings.cpp:167-260: signed packed-int4 weights [N, K/2] (even k in the low
    nibble), per-channel weight scale, per-token activation scale, fused epilogue.
    The tcgen05 kernel takes K % 32 == 0 and N % 8 == 0; other shapes allowed by the
    reference (K % 4 == 0, any N) are zero-padded here, as the reference pads its
    N tail (bindings.cpp:229-255).  From W4_WIDEN_MIN_ROWS rows on, the weight is widened
    to int8 once and the W8A8 GEMM runs (identical results: the contraction is exact)."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = activation_scale.to(torch.float32).contiguous()
    weight_scale = weight_scale.to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    if activation.dtype != torch.int8:
        raise RuntimeError("activation must be int8")
    if weight.dtype != torch.int8:
        raise RuntimeError("weight must be packed int8 storage")
    dev = activation.device
    if weight.device != dev:
        raise RuntimeError("activation and weight must be on the same CUDA device")
    if not (activation_scale.is_cuda and weight_scale.is_cuda):
        raise RuntimeError("scales must be CUDA tensors")
    if activation_scale.device != dev or weight_scale.device != dev:
        raise RuntimeError("scales must be on the activation device")
    m, k = activation.shape
    n = weight.shape[0]
    if k % 4 != 0:
        raise RuntimeError("activation K must be divisible by 4")
    if weight.shape[1] * 2 != k:
        raise RuntimeError("packed weight K must match activation K")
    if activation_scale.numel() != m:
        raise RuntimeError("activation_scale must contain one value per row")
    if weight_scale.numel() != n:
        raise RuntimeError("weight_scale must contain one value per output channel")
    if bias is not None and (not bias.is_cuda or bias.device != dev):
        raise RuntimeError("bias must be on the activation device")
    if bias is not None and bias.numel() != n:
        raise RuntimeError("bias must contain one value per output channel")
    weight_scale = weight_scale.reshape(-1)
    bias = None if bias is None else bias.reshape(-1)
    k_pad = -(-k // 32) * 32
    n_pad = -(-n // 8) * 8
    if k_pad != k:
        activation = torch.nn.functional.pad(activation, (0, k_pad - k))
        weight = torch.nn.functional.pad(weight, (0, (k_pad - k) // 2))
    if n_pad != n:
        weight = torch.nn.functional.pad(weight, (0, 0, 0, n_pad - n))
        weight_scale = torch.nn.functional.pad(weight_scale, (0, n_pad - n))
        if bias is not None:
            bias = torch.nn.functional.pad(bias, (0, n_pad - n))
    out = torch.empty((m, n_pad), dtype=torch.bfloat16, device=dev)
    if m == 0 or n == 0:
        return out[:, :n]
    activation, weight = _aligned(activation), _aligned(weight)
    with torch.cuda.device(dev):
        if m >= W4_WIDEN_MIN_ROWS:
            wide = _widen_s4(weight)
            _lib.check(_lib.load().ctu_int8_linear(
                _ptr(activation), _ptr(wide), _ptr(activation_scale), _ptr(weight_scale), n_pad,
                _ptr(bias), _ptr(out), m, n_pad, k_pad, _stream(dev)))
        else:
            _lib.check(_lib.load().ctu_w4a8_linear(
                _ptr(activation), _ptr(weight), _ptr(activation_scale), _ptr(weight_scale), n_pad,
                _ptr(bias), _ptr(out), m, n_pad, k_pad, _stream(dev)))
    return out if n_pad == n else out[:, :n].contiguous()


# Decoded-weight workspace cap of the B200 codebook path: the whole output dimension is
# decoded at once (one tensor-core GEMM) whenever its int8 weights fit in this budget.
CODEBOOK_WORKSPACE_BYTES = 256 << 20
# Reference chunk of the staged path (dispatch.py TURING_CODEBOOK_W4A8_CHUNK_ROWS).
TURING_CODEBOOK_W4A8_CHUNK_ROWS = 4096


def _codebook_chunk_rows(m: int, n: int, k: int, group_size: int, chunk_rows: int) -> int:
    """bindings.cpp:328-350 policy, B200 sizes.  -1 (force the inline decode) keeps the
    reference's precondition; its B200 form decodes all N at once like chunk_rows=0.
    0 decodes as many channels as the workspace budget allows; a positive multiple of 8
    forces that chunk."""
    if chunk_rows < -1:
        raise RuntimeError("chunk_rows must be -1, 0, or a positive multiple of 8")
    if chunk_rows == -1 and not (group_size == 16 and m > 8192):
        raise RuntimeError("forced inline codebook W4A8 requires group_size=16 and M>8192")
    if chunk_rows > 0:
        if chunk_rows % 8 != 0:
            raise RuntimeError("chunk_rows must be divisible by 8")
        return min(n, chunk_rows)
    budget_rows = max(8, (CODEBOOK_WORKSPACE_BYTES // max(k, 1)) // 8 * 8)
    return min(n, budget_rows)


def turing_codebook_w4a8_linear(activation, weight, activation_scale, group_scale, channel_scale, codebook,
                                bias=None, group_size=16, chunk_rows=0, tile_policy=0):
    """bindings.cpp:262-370: grouped-codebook W4A8 (4-bit codes [N, K/2], e4m3fn group
    scales [N, K/group_size], 16-entry fp32 codebook, per-channel fp32 scale)."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = activation_scale.reshape(-1).to(torch.float32).contiguous()
    group_scale = group_scale.contiguous()
    channel_scale = channel_scale.reshape(-1).to(torch.float32).contiguous()
    codebook = codebook.reshape(-1).to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(torch.float32).contiguous()
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check_cuda_2d(group_scale, "group_scale")
    if activation.dtype != torch.int8:
        raise RuntimeError("activation must be int8")
    if weight.dtype != torch.int8:
        raise RuntimeError("weight must use packed int8 storage")
    if group_scale.dtype == torch.float8_e4m3fn:
        group_scale = group_scale.view(torch.uint8)
    if group_scale.dtype != torch.uint8:
        raise RuntimeError("group_scale must contain raw float8_e4m3fn bytes")
    dev = activation.device
    if any(t.device != dev for t in (weight, group_scale, activation_scale, channel_scale, codebook)):
        raise RuntimeError("all codebook W4A8 tensors must use the same CUDA device")
    m, k = activation.shape
    n = weight.shape[0]
    if m <= 0 or n <= 0 or k <= 0:
        raise RuntimeError("codebook W4A8 dimensions must be positive")
    if k % 16 != 0 or n % 8 != 0:
        raise RuntimeError("codebook W4A8 requires K divisible by 16 and N divisible by 8")
    if weight.shape[1] * 2 != k:
        raise RuntimeError("packed weight K must match activation K")
    if not (group_size >= 4 and k % group_size == 0 and (16 % group_size == 0 or group_size % 16 == 0)):
        raise RuntimeError("unsupported codebook W4A8 group_size")
    if tuple(group_scale.shape) != (n, k // group_size):
        raise RuntimeError("group_scale must have shape [N, K/group_size]")
    if activation_scale.numel() != m:
        raise RuntimeError("activation_scale must contain one value per activation row")
    if channel_scale.numel() != n:
        raise RuntimeError("channel_scale must contain one value per output channel")
    if codebook.numel() != 16:
        raise RuntimeError("codebook must contain 16 float32 values")
    if bias is not None and (not bias.is_cuda or bias.device != dev):
        raise RuntimeError("bias must use the activation CUDA device")
    if bias is not None and bias.numel() != n:
        raise RuntimeError("bias must contain one value per output channel")
    rows = _codebook_chunk_rows(m, n, k, int(group_size), int(chunk_rows))
    workspace = torch.empty((rows, k), dtype=torch.int8, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    activation, weight = _aligned(activation), _aligned(weight)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ctu_codebook_w4a8_linear(
            _ptr(activation), _ptr(weight), _ptr(activation_scale), _ptr(group_scale), _ptr(channel_scale),
            _ptr(codebook), _ptr(bias), _ptr(out), _ptr(workspace), rows, m, n, k, int(group_size), _stream(dev)))
    return out


def codebook_decode_s8(weight, group_scale, codebook, group_size=16):
    """The codebook weight decode alone (w4a8.cu:903-976): int8 [N, K]."""
    weight = _aligned(weight.contiguous())
    if group_scale.dtype == torch.float8_e4m3fn:
        group_scale = group_scale.view(torch.uint8)
    group_scale = group_scale.contiguous()
    codebook = codebook.reshape(-1).to(torch.float32).contiguous()
    n, k = weight.shape[0], 2 * weight.shape[1]
    out = torch.empty((n, k), dtype=torch.int8, device=weight.device)
    with torch.cuda.device(weight.device):
        _lib.check(_lib.load().ctu_codebook_decode_s8(
            _ptr(weight), _ptr(group_scale), _ptr(codebook), _ptr(out), n, k, int(group_size), _stream(weight.device)))
    return out


def turing_dequantize_int8_bf16(accumulator, activation_scale, weight_scale, output_columns=-1):
    """bindings.cpp:423-472."""
    accumulator = accumulator.contiguous()
    activation_scale = activation_scale.reshape(-1).to(torch.float32).contiguous()
    weight_scale = weight_scale.reshape(-1).to(torch.float32).contiguous()
    _check_cuda_2d(accumulator, "accumulator")
    if accumulator.dtype != torch.int32:
        raise RuntimeError("accumulator must be int32")
    if not (activation_scale.is_cuda and weight_scale.is_cuda):
        raise RuntimeError("scales must be CUDA tensors")
    if activation_scale.device != accumulator.device or weight_scale.device != accumulator.device:
        raise RuntimeError("accumulator and scales must use the same CUDA device")
    rows, acc_cols = accumulator.shape
    if output_columns < 0:
        output_columns = acc_cols
    if rows <= 0 or acc_cols <= 0:
        raise RuntimeError("INT8 BF16 epilogue dimensions must be positive")
    if output_columns <= 0 or output_columns > acc_cols:
        raise RuntimeError("output_columns must be positive and no larger than the accumulator width")
    if activation_scale.numel() != rows:
        raise RuntimeError("activation_scale must contain one value per accumulator row")
    if weight_scale.numel() not in (1, output_columns):
        raise RuntimeError("weight_scale must be scalar or contain one value per output column")
    out = torch.empty((rows, output_columns), dtype=torch.bfloat16, device=accumulator.device)
    with torch.cuda.device(accumulator.device):
        _lib.check(_lib.load().ctu_dequantize_int8_bf16(
            _ptr(accumulator), acc_cols, _ptr(activation_scale), _ptr(weight_scale), weight_scale.numel(),
            _ptr(out), rows, output_columns, _stream(accumulator.device)))
    return out


_NORM_TYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _check_float_like(t: torch.Tensor, name: str) -> None:
    if t.dtype not in _NORM_TYPES:
        raise RuntimeError(f"{name} must be float16, bfloat16, or float32")


def turing_segmented_rms_adaln(input, weight, scale, shift, segments, epsilon=1.0e-5):
    """bindings.cpp:767-834: affine RMSNorm + segmented AdaLN, output like ``input``."""
    input = input.contiguous()
    weight = weight.contiguous()
    segments = segments.contiguous()
    _check_cuda_2d(input, "input")
    _check_float_like(input, "input")
    if not (weight.is_cuda and weight.dim() == 1 and weight.is_contiguous()):
        raise RuntimeError("weight must be a contiguous 1D CUDA tensor")
    if not (scale.is_cuda and scale.dim() == 2 and scale.stride(1) == 1):
        raise RuntimeError("scale must be a CUDA matrix with contiguous rows")
    if not (shift.is_cuda and shift.dim() == 2 and shift.stride(1) == 1):
        raise RuntimeError("shift must be a CUDA matrix with contiguous rows")
    if not (segments.is_cuda and segments.dim() == 2 and segments.is_contiguous()):
        raise RuntimeError("segments must be a contiguous 2D CUDA tensor")
    if segments.dtype != torch.int32 or segments.size(1) != 3:
        raise RuntimeError("segments must be int32 [start, stop, modulation_row] triples")
    dev = input.device
    if not (weight.device == dev and scale.device == dev and shift.device == dev and segments.device == dev):
        raise RuntimeError("all segmented RMSNorm+AdaLN tensors must use the same CUDA device")
    if not (weight.dtype == input.dtype and scale.dtype == input.dtype and shift.dtype == input.dtype):
        raise RuntimeError("weight, scale, and shift dtypes must match input")
    rows, hidden = input.shape
    if rows <= 0 or hidden <= 0:
        raise RuntimeError("segmented RMSNorm+AdaLN input dimensions must be positive")
    if weight.numel() != hidden:
        raise RuntimeError("RMSNorm weight length must match the input hidden dimension")
    if scale.size(0) <= 0 or scale.size(1) != hidden:
        raise RuntimeError("scale must be [modulation_rows, hidden]")
    if shift.shape != scale.shape:
        raise RuntimeError("shift shape must match scale shape")
    if segments.size(0) <= 0:
        raise RuntimeError("segments must contain at least one row")
    limit = 2**31 - 1
    if rows > limit or hidden > limit or scale.stride(0) > limit or shift.stride(0) > limit:
        raise RuntimeError("segmented RMSNorm+AdaLN dimensions exceed the CUDA kernel range")
    if not (math.isfinite(epsilon) and epsilon > 0.0):
        raise RuntimeError("RMSNorm epsilon must be finite and positive")
    out = torch.empty_like(input)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ctu_segmented_rms_adaln(
            _ptr(input), _ptr(weight), _ptr(scale), scale.stride(0), _ptr(shift), shift.stride(0), _ptr(segments),
            segments.size(0), _ptr(out), rows, hidden, scale.size(0), float(epsilon), _NORM_TYPES[input.dtype],
            _stream(dev)))
    return out


def turing_layer_norm_adaln(input, scale, shift, epsilon=1.0e-5):
    """bindings.cpp:836-880: LayerNorm (fp32 Welford statistics) + Wan AdaLN."""
    input = input.contiguous()
    scale = scale.contiguous()
    shift = shift.contiguous()
    if not (input.is_cuda and input.dim() == 3):
        raise RuntimeError("input must be contiguous CUDA [batch, sequence, hidden]")
    _check_float_like(input, "input")
    if not (scale.is_cuda and scale.dim() == 3):
        raise RuntimeError("scale must be contiguous CUDA [batch, modulation_steps, hidden]")
    if not (shift.is_cuda and shift.dim() == 3):
        raise RuntimeError("shift must be contiguous CUDA [batch, modulation_steps, hidden]")
    if not (input.device == scale.device and input.device == shift.device):
        raise RuntimeError("LayerNorm+AdaLN tensors must use the same CUDA device")
    if not (input.dtype == scale.dtype and input.dtype == shift.dtype):
        raise RuntimeError("LayerNorm+AdaLN tensor dtypes must match")
    if scale.shape != shift.shape:
        raise RuntimeError("shift shape must match scale shape")
    if scale.size(0) != input.size(0) or scale.size(2) != input.size(2):
        raise RuntimeError("scale must match input batch and hidden dimensions")
    batch, sequence, hidden = input.shape
    if batch <= 0 or sequence <= 0 or hidden <= 0 or scale.size(1) <= 0:
        raise RuntimeError("LayerNorm+AdaLN dimensions must be positive")
    limit = 2**31 - 1
    if batch * sequence > limit or sequence > limit or hidden > limit or scale.size(1) > limit:
        raise RuntimeError("LayerNorm+AdaLN dimensions exceed the CUDA kernel range")
    if not (math.isfinite(epsilon) and epsilon > 0.0):
        raise RuntimeError("LayerNorm epsilon must be finite and positive")
    out = torch.empty_like(input)
    with torch.cuda.device(input.device):
        _lib.check(_lib.load().ctu_layer_norm_adaln(
            _ptr(input), _ptr(scale), _ptr(shift), _ptr(out), batch, sequence, hidden, scale.size(1),
            float(epsilon), _NORM_TYPES[input.dtype], _stream(input.device)))
    return out


# ----------------------------------------------------------------------------- B200 extras
def int4_linear(qactivation, qweight, activation_scale, wscales, bias=None, out_dtype=torch.bfloat16):
    """W4A4 GEMM: packed signed-int4 ConvRot codes [M, K/2] x packed signed-int4 weights
    [N, K/2], per-token activation scale, per-channel weight scale (the 1-D ``wscales``
    the plugin registry requires, dispatch.py:1031-1034), optional bias; same fused
    epilogue as int8_linear.  Stands in for comfy-kitchen's ``int4_linear`` that
    ``convrot_w4a4_linear(linear_dtype="int4")`` calls (dispatch.py:927-934).  From
    W4_WIDEN_MIN_ROWS rows on, both operands are widened to int8 and the W8A8 GEMM runs."""
    qactivation = qactivation.contiguous()
    qweight = qweight.contiguous()
    activation_scale = activation_scale.reshape(-1).to(torch.float32).contiguous()
    wscales = wscales.reshape(-1).to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(torch.float32).contiguous()
    _check_cuda_2d(qactivation, "activation")
    _check_cuda_2d(qweight, "weight")
    if qactivation.dtype != torch.int8 or qweight.dtype != torch.int8:
        raise RuntimeError("W4A4 activation and weight must use packed int8 storage")
    dev = qactivation.device
    m, kp = qactivation.shape
    n = qweight.shape[0]
    k = 2 * kp
    if qweight.shape[1] != kp:
        raise RuntimeError("W4A4 packed K dimensions must match")
    if activation_scale.numel() != m:
        raise RuntimeError("activation_scale must contain one value per row")
    if wscales.numel() not in (1, n):
        raise RuntimeError("wscales must be scalar or contain one value per output channel")
    if bias is not None and bias.numel() != n:
        raise RuntimeError("bias must contain one value per output channel")
    k_pad = -(-k // 32) * 32
    n_pad = -(-n // 8) * 8
    if k_pad != k:
        qactivation = torch.nn.functional.pad(qactivation, (0, (k_pad - k) // 2))
        qweight = torch.nn.functional.pad(qweight, (0, (k_pad - k) // 2))
    if wscales.numel() == 1:
        wscales = wscales.expand(n).contiguous()
    if n_pad != n:
        qweight = torch.nn.functional.pad(qweight, (0, 0, 0, n_pad - n))
        wscales = torch.nn.functional.pad(wscales, (0, n_pad - n))
        if bias is not None:
            bias = torch.nn.functional.pad(bias, (0, n_pad - n))
    out = torch.empty((m, n_pad), dtype=torch.bfloat16, device=dev)
    if m > 0 and n > 0:
        with torch.cuda.device(dev):
            if m >= W4_WIDEN_MIN_ROWS:
                a8, w8 = _widen_s4(qactivation), _widen_s4(qweight)
                _lib.check(_lib.load().ctu_int8_linear(
                    _ptr(a8), _ptr(w8), _ptr(activation_scale), _ptr(wscales), n_pad,
                    _ptr(bias), _ptr(out), m, n_pad, k_pad, _stream(dev)))
            else:
                _lib.check(_lib.load().ctu_w4a4_linear(
                    _ptr(_aligned(qactivation)), _ptr(_aligned(qweight)), _ptr(activation_scale), _ptr(wscales),
                    n_pad, _ptr(bias), _ptr(out), m, n_pad, k_pad, _stream(dev)))
    out = out if n_pad == n else out[:, :n].contiguous()
    return out if out_dtype == torch.bfloat16 else out.to(out_dtype)


# Per-group (128 along K) formats.  The reference has no kernel or checkpoint layout for
# them (its W4A4 path, dispatch.py:876-936, hands int4 activations to comfy-kitchen's
# int4_linear with 64-column weight groups; its asym_w4a8_int8 format is the grouped
# codebook); the arithmetic is this library's (see ctu_b200.h).
QUANT_GROUP = 128


def bf16_int4_g128_convrot_quantize(input, group_size=256):
    """ConvRot rotation, then int4 codes with one scale per token and 128 columns:
    ``(codes int8 [M, K/2] packed, scales fp32 [M, K/128])``.  ``group_size`` is the
    rotation block: 256 (the reference's rotation) or 128 (this library's block-128
    rotation, see ctu_b200.h)."""
    x = input.contiguous()
    _check_cuda_2d(x, "input")
    if x.dtype != torch.bfloat16:
        raise RuntimeError("per-group INT4 ConvRot input must be bfloat16")
    if group_size not in (128, 256):
        raise RuntimeError("per-group INT4 ConvRot supports group_size=256 or 128")
    rows, k = x.shape
    if rows <= 0 or k <= 0 or k % 256 != 0:
        raise RuntimeError("per-group INT4 ConvRot width must be positive and divisible by 256")
    x = _aligned(x)
    codes = torch.empty((rows, k // 2), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, k // QUANT_GROUP), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        fn = (_lib.load().ctu_convrot_quantize_int4_g128_b128 if group_size == 128
              else _lib.load().ctu_convrot_quantize_int4_g128)
        _lib.check(fn(_ptr(x), rows, k, _ptr(codes), _ptr(scales), _stream(x.device)))
    return codes, scales


def _group_major_scales(w_scale: torch.Tensor, n: int, groups: int) -> torch.Tensor:
    """Checkpoint weight scales [N, K/128] (fp16) -> fp32 [K/128, N], group-major."""
    if w_scale.shape != (n, groups):
        raise RuntimeError(f"weight_scale must have shape [{n}, {groups}]")
    return w_scale.to(torch.float16).to(torch.float32).t().contiguous()


def _grouped_common(m, n, k, bias, dev):
    if k % QUANT_GROUP != 0 or n % 8 != 0:
        raise RuntimeError(f"per-group linears require K%128=0 and N%8=0 (got K={k}, N={n})")
    if bias is not None:
        bias = bias.reshape(-1).to(torch.float32).contiguous()
        if bias.numel() != n:
            raise RuntimeError("bias must contain one value per output channel")
    return bias, torch.empty((m, n), dtype=torch.bfloat16, device=dev)


def asym_w4a8_g128_linear(activation, weight, activation_scale, weight_scale, weight_zero, bias=None):
    """Asymmetric uint4 W4A8: int8 activations [M, K] with per-token scales; uint4
    weights packed [N, K/2] (uint8 storage, even column in the low nibble) with an fp16
    scale and a uint4 zero point per 128 columns ([N, K/128] each) -> bf16 [M, N]."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    if activation.dtype != torch.int8:
        raise RuntimeError("asymmetric W4A8 activation must be int8")
    if weight.dtype not in (torch.uint8, torch.int8):
        raise RuntimeError("asymmetric W4A8 weight must use packed uint8 storage")
    dev = activation.device
    m, k = activation.shape
    n = weight.shape[0]
    if weight.shape[1] * 2 != k:
        raise RuntimeError("asymmetric W4A8 packed weight must have K/2 columns")
    bias, out = _grouped_common(m, n, k, bias, dev)
    groups = k // QUANT_GROUP
    w_scale = _group_major_scales(weight_scale, n, groups)
    if weight_zero.shape != (n, groups):
        raise RuntimeError(f"weight_zero must have shape [{n}, {groups}]")
    w_zero = weight_zero.to(torch.uint8).contiguous()
    a_scale = activation_scale.reshape(-1).to(torch.float32).contiguous()
    if a_scale.numel() != m:
        raise RuntimeError("activation_scale must contain one value per row")
    if m > 0 and n > 0:
        workspace = torch.empty((n, k), dtype=torch.int8, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.load().ctu_asym_w4a8_g128_linear(
                _ptr(_aligned(activation)), _ptr(_aligned(weight)), _ptr(a_scale), _ptr(w_scale), _ptr(w_zero),
                _ptr(bias), _ptr(out), _ptr(workspace), m, n, k, _stream(dev)))
    return out


def w4a4_g128_linear(qactivation, qweight, activation_scale, weight_scale, bias=None):
    """W4A4 with per-token-per-group activation scales: packed signed int4 activations
    [M, K/2] with fp32 scales [M, K/128] (bf16_int4_g128_convrot_quantize), packed signed
    int4 weights [N, K/2] with fp16 scales [N, K/128] -> bf16 [M, N]."""
    qactivation = qactivation.contiguous()
    qweight = qweight.contiguous()
    _check_cuda_2d(qactivation, "activation")
    _check_cuda_2d(qweight, "weight")
    if qactivation.dtype != torch.int8 or qweight.dtype != torch.int8:
        raise RuntimeError("W4A4 activation and weight must use packed int8 storage")
    dev = qactivation.device
    m, kp = qactivation.shape
    n = qweight.shape[0]
    k = 2 * kp
    if qweight.shape[1] != kp:
        raise RuntimeError("W4A4 packed K dimensions must match")
    bias, out = _grouped_common(m, n, k, bias, dev)
    groups = k // QUANT_GROUP
    w_scale = _group_major_scales(weight_scale, n, groups)
    a_scale = activation_scale.to(torch.float32).contiguous()
    if a_scale.shape != (m, groups):
        raise RuntimeError(f"activation_scale must have shape [{m}, {groups}]")
    if m > 0 and n > 0:
        a_ws = torch.empty((m, k), dtype=torch.int8, device=dev)
        w_ws = torch.empty((n, k), dtype=torch.int8, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.load().ctu_w4a4_g128_linear(
                _ptr(_aligned(qactivation)), _ptr(_aligned(qweight)), _ptr(a_scale), _ptr(w_scale), _ptr(bias),
                _ptr(out), _ptr(a_ws), _ptr(w_ws), m, n, k, _stream(dev)))
    return out


def int8_gemm_s32(activation, weight, out=None):
    """Exact int32 accumulators ``activation @ weight.T`` (no epilogue)."""
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    m, k = activation.shape
    n = weight.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.int32, device=activation.device)
    with torch.cuda.device(activation.device):
        _lib.check(_lib.load().ctu_int8_gemm_s32(
            _ptr(_aligned(activation)), _ptr(_aligned(weight)), _ptr(out), out.stride(0), m, n, k,
            _stream(activation.device)))
    return out
