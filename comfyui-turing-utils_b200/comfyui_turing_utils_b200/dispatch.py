"""Plugin-facing ConvRot linear entry points on B200, without comfy-kitchen.

Mirrors the functions of the reference plugin's dispatcher that comfy-kitchen's
registry and the model adapters call for the ConvRot quantized linear
(comfyui_turing_utils/quantization/dispatch.py): same names, argument names and
defaults, same flattening of leading dimensions and scale normalisation.  Where the
reference delegates to comfy-kitchen (a configuration its fast path does not take:
non-bf16 input, ConvRot off, group size other than 256, unknown fused activations)
this module raises NotImplementedError instead, because kitchen is not part of the
B200 build and there is no CPU or eager fallback.
"""

from __future__ import annotations

import torch

import comfyui_turing_utils_kernel as ops
from comfyui_turing_utils_kernel import _C

CONVROT_GROUP = 256
_FUSED_ACTS = (None, "none", "swiglu", "gelu_tanh")

BACKEND_NAME = "turing_utils_sm75"  # the registry name the plugin's callers look up (dispatch.py:19)
# Reference decode chunk of the staged codebook path (dispatch.py:26); kept for planning callers.
TURING_CODEBOOK_W4A8_CHUNK_ROWS = 4096
_PREFLIGHTED_DEVICES: set[int] = set()
_PREFLIGHTED_CODEBOOK_DEVICES: set[int] = set()


def turing_int8_workspace_bytes(rows: int, output_channels: int) -> int:
    """dispatch.py:32-43: global int32 workspace of the selected W8A8 path.  The B200 GEMM
    fuses the epilogue at every size and never stages int32 accumulators: 0."""
    return 0


def turing_codebook_w4a8_workspace_bytes(input_channels: int, output_channels: int) -> int:
    """dispatch.py:46-56: decoded-weight workspace of grouped W4A8.  The B200 op decodes
    all output channels at once while they fit 256 MiB (``_C.CODEBOOK_WORKSPACE_BYTES``),
    else in 8-row-aligned chunks of that size."""
    if input_channels <= 0 or output_channels <= 0:
        return 0
    rows = _C._codebook_chunk_rows(1, int(output_channels), int(input_channels), 16, 0)
    return rows * int(input_channels)


def convrot_swiglu_channel_sharding_available() -> bool:
    """dispatch.py:67-69: exact two-pass SwiGLU channel streaming is in the ABI."""
    return hasattr(_C, "turing_swiglu_int8_convrot_quantize_scaled")


def quantize_convrot_swiglu_with_scale(x: torch.Tensor, scale: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """dispatch.py:450-465: one SwiGLU channel shard quantized with whole-row scales."""
    return ops.turing_swiglu_int8_convrot_quantize_scaled(x.contiguous(), scale.reshape(-1).contiguous(),
                                                          int(group_size))


def _require(condition: bool, what: str) -> None:
    if not condition:
        raise NotImplementedError(
            f"{what}: the reference hands this case to comfy-kitchen, which the B200 build does not include")


def _quantize_int8(x2d: torch.Tensor, group_size: int, input_act: str | None):
    """dispatch.py:343-414 without kitchen: every width uses the fused kernel."""
    if input_act not in _FUSED_ACTS:
        raise ValueError(f"unsupported fused INT8 activation: {input_act!r}")
    if input_act == "gelu_tanh":
        return ops.turing_bf16_gelu_int8_convrot_quantize(x2d, group_size)
    return ops.turing_bf16_int8_convrot_quantize(x2d, group_size, swiglu=input_act == "swiglu")


def _quantize_int4(x2d: torch.Tensor, group_size: int, input_act: str | None):
    """dispatch.py:468-556 without kitchen."""
    if input_act not in _FUSED_ACTS:
        raise ValueError(f"unsupported fused INT4 activation: {input_act!r}")
    if input_act == "gelu_tanh":
        return ops.turing_bf16_gelu_int4_convrot_quantize(x2d, group_size)
    if input_act == "swiglu" and x2d.shape[1] % 2 != 0:
        raise ValueError("SwiGLU input width must be even")
    return ops.turing_bf16_int4_convrot_quantize(x2d, group_size, swiglu=input_act == "swiglu")


def quantize_convrot_int8_activation(x: torch.Tensor, group_size: int = 256):
    """dispatch.py:417-429: quantize a 2D bf16 activation once for reuse by several GEMMs."""
    if x.ndim != 2:
        raise ValueError("ConvRot W8 activation must be two-dimensional")
    if x.dtype is not torch.bfloat16:
        raise ValueError("ConvRot W8 activation must use BF16 storage")
    if not x.is_cuda:
        raise ValueError("ConvRot W8 activation must be on CUDA")
    return _quantize_int8(x.contiguous(), int(group_size), None)


def quantize_convrot_swiglu_activation(x: torch.Tensor, group_size: int = 256):
    """dispatch.py:432-446: fused SwiGLU + ConvRot quantization of a [M, 2K] tile."""
    if x.ndim != 2 or x.shape[1] % 2:
        raise ValueError("SwiGLU ConvRot input must be 2D [M, 2K]")
    if x.dtype is not torch.bfloat16:
        raise ValueError("SwiGLU ConvRot input must use BF16 storage")
    if not x.is_cuda:
        raise ValueError("SwiGLU ConvRot input must be on CUDA")
    return ops.turing_bf16_int8_convrot_quantize(x.contiguous(), int(group_size), swiglu=True)


def _int8_gemm(qactivation, weight, activation_scale, weight_scale, bias, output_dtype):
    """dispatch.py:616-720: normalise scales, then the fused tcgen05 GEMM (no int32
    workspace at any size; the reference's cuBLAS/kitchen branches are not needed)."""
    m, k = qactivation.shape
    n = weight.shape[0]
    activation_scale = activation_scale.to(device=qactivation.device, dtype=torch.float32).reshape(-1).contiguous()
    weight_scale = weight_scale.to(device=qactivation.device, dtype=torch.float32).reshape(-1).contiguous()
    if activation_scale.numel() != m:
        raise ValueError(f"W8A8 activation scale must have {m} values, got {activation_scale.numel()}")
    if weight_scale.numel() not in (1, n):
        raise ValueError(f"W8A8 weight scale must be scalar or have {n} values, got {weight_scale.numel()}")
    if weight_scale.numel() == 1:
        weight_scale = weight_scale.expand(n).contiguous()
    if bias is not None:
        bias = bias.to(device=qactivation.device, dtype=torch.float32)
    output = ops.turing_int8_linear(qactivation, weight, activation_scale, weight_scale, bias)
    return output if output_dtype == torch.bfloat16 else output.to(output_dtype)


def int8_linear_from_quantized(
    qactivation: torch.Tensor,
    activation_scale: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """dispatch.py:723-745: W8 GEMM from an activation quantized once by the caller."""
    if qactivation.ndim != 2 or weight.ndim != 2:
        raise ValueError("quantized W8 linear expects two-dimensional tensors")
    if qactivation.dtype is not torch.int8 or weight.dtype is not torch.int8:
        raise ValueError("quantized W8 linear expects INT8 activation and weight")
    if qactivation.shape[1] != weight.shape[1]:
        raise ValueError("quantized W8 activation and weight widths differ")
    return _int8_gemm(qactivation, weight.contiguous(), activation_scale, weight_scale, bias, out_dtype)


def int8_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
    convrot: bool = False,
    convrot_groupsize: int = 256,
    input_act: str | None = None,
) -> torch.Tensor:
    """dispatch.py:748-800: ConvRot W8A8 linear over [..., K] bf16 activations."""
    _require(x.dtype == torch.bfloat16, "non-bf16 activations")
    _require(bool(convrot), "INT8 linear without ConvRot")
    _require(convrot_groupsize == CONVROT_GROUP, f"ConvRot group size {convrot_groupsize}")
    _require(input_act in _FUSED_ACTS, f"input activation {input_act!r}")
    original_shape = x.shape
    x2d = x.reshape(-1, original_shape[-1]).contiguous()
    if input_act is None and weight.ndim == 2 and weight.shape[1] == x2d.shape[1]:
        # Plain rows: one library call (the fused quantizer + GEMM kernel where it pays).
        n = weight.shape[0]
        weight_scale = weight_scale.to(device=x2d.device, dtype=torch.float32).reshape(-1).contiguous()
        if weight_scale.numel() not in (1, n):
            raise ValueError(f"W8A8 weight scale must be scalar or have {n} values, got {weight_scale.numel()}")
        if weight_scale.numel() == 1:
            weight_scale = weight_scale.expand(n).contiguous()
        if bias is not None:
            bias = bias.to(device=x2d.device, dtype=torch.float32)
        output = ops.turing_convrot_int8_linear(x2d, weight.contiguous(), weight_scale, bias, convrot_groupsize)
        dtype = out_dtype or x.dtype
        output = output if dtype == torch.bfloat16 else output.to(dtype)
    else:
        qactivation, activation_scale = _quantize_int8(x2d, convrot_groupsize, input_act)
        output = _int8_gemm(qactivation, weight.contiguous(), activation_scale, weight_scale, bias,
                            out_dtype or x.dtype)
    return output.reshape(*original_shape[:-1], weight.shape[0])


def codebook_w4a8_linear(
    x: torch.Tensor,
    qdata: torch.Tensor,
    s_rel: torch.Tensor,
    s_channel: torch.Tensor,
    codebook: torch.Tensor | None = None,
    correction: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    group_size: int = 16,
    convrot_groupsize: int = 256,
    out_dtype: torch.dtype = torch.bfloat16,
    input_act: str | None = None,
) -> torch.Tensor:
    """dispatch.py:803-869: grouped-codebook W4A8 on the fast path's conditions."""
    _require(x.dtype == torch.bfloat16 and out_dtype == torch.bfloat16, "non-bf16 activations or output")
    _require(convrot_groupsize == CONVROT_GROUP, f"ConvRot group size {convrot_groupsize}")
    _require(correction is None, "a codebook correction term")
    _require(codebook is not None and codebook.numel() == 16, "a codebook without 16 entries")
    _require(s_rel.dtype == torch.float8_e4m3fn, "non-e4m3 group scales")
    _require(qdata.ndim == 2 and qdata.shape[0] % 8 == 0 and qdata.shape[1] * 2 == x.shape[-1],
             "this packed weight shape")
    _require(input_act in _FUSED_ACTS, f"input activation {input_act!r}")
    original_shape = x.shape
    x2d = x.reshape(-1, original_shape[-1]).contiguous()
    qactivation, activation_scale = _quantize_int8(x2d, convrot_groupsize, input_act)
    output = ops.turing_codebook_w4a8_linear(qactivation, qdata, activation_scale, s_rel, s_channel, codebook, bias,
                                             group_size)
    return output.reshape(*original_shape[:-1], qdata.shape[0])


# Kitchen resolves backend implementations by the public capability name (dispatch.py:872-873).
w4a8_int8_linear = codebook_w4a8_linear


# dispatch.py:873: the name comfy-kitchen's registry calls for the grouped-codebook format.
w4a8_int8_linear = codebook_w4a8_linear


def convrot_w4a4_linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    wscales: torch.Tensor,
    bias: torch.Tensor | None = None,
    convrot_groupsize: int = 256,
    quant_group_size: int = 64,
    linear_dtype: str = "int4",
    input_act: str | None = None,
) -> torch.Tensor:
    """dispatch.py:876-936: W4 weights with int8 (W4A8) or int4 (W4A4) activations."""
    _require(linear_dtype in {"int4", "int8"}, f"linear_dtype {linear_dtype!r}")
    _require(convrot_groupsize == CONVROT_GROUP, f"ConvRot group size {convrot_groupsize}")
    _require(quant_group_size == 64, f"quant_group_size {quant_group_size}")
    _require(x.dtype == torch.bfloat16, "non-bf16 activations")
    _require(input_act in _FUSED_ACTS, f"input activation {input_act!r}")
    original_shape = x.shape
    x2d = x.reshape(-1, original_shape[-1]).contiguous()
    if linear_dtype == "int8":
        qactivation, activation_scale = _quantize_int8(x2d, convrot_groupsize, input_act)
        output = ops.turing_w4a8_linear(qactivation, qweight, activation_scale, wscales, bias)
    else:
        qactivation, activation_scale = _quantize_int4(x2d, convrot_groupsize, input_act)
        output = _C.int4_linear(qactivation, qweight.contiguous(), activation_scale, wscales, bias, out_dtype=x.dtype)
    return output.reshape(*original_shape[:-1], qweight.shape[0])


def is_supported_b200_device(device: torch.device) -> bool:
    """The device check the preflights make (dispatch.py:89 checks for a Turing tensor-core
    device): a CUDA device of compute capability 10.0, the only arch libctu_b200.so holds."""
    if device.type != "cuda" or not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(device) == (10, 0)


def preflight_w4a8(device: torch.device) -> None:
    """dispatch.py:88-150: once per device, a numerical self-test of the signed W4A8 op and
    of the ConvRot W4A8 linear (K = 256 and 8192, and a fused SwiGLU input)."""
    if not is_supported_b200_device(device):
        raise RuntimeError(f"unsupported device {device}")
    if not hasattr(_C, "turing_w4a8_linear"):
        raise RuntimeError("the installed comfyui-turing-utils-kernel does not provide W4A8")
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index in _PREFLIGHTED_DEVICES:
        return
    activation = ((torch.arange(3 * 64, device=device) % 23) - 11).to(torch.int8).reshape(3, 64)
    weight_values = ((torch.arange(5 * 64, device=device) % 15) - 7).to(torch.int8).reshape(5, 64)
    packed = ((weight_values[:, 0::2].to(torch.int32) & 0x0F) | ((weight_values[:, 1::2].to(torch.int32) & 0x0F) << 4)
              ).to(torch.int8)
    a_s = torch.linspace(0.01, 0.03, 3, device=device)
    w_s = torch.linspace(0.02, 0.06, 5, device=device)
    bias = torch.linspace(-0.2, 0.2, 5, dtype=torch.bfloat16, device=device)
    out = ops.turing_w4a8_linear(activation, packed, a_s, w_s, bias)
    ref = (activation.float() @ weight_values.float().t()) * a_s[:, None] * w_s[None, :] + bias.float()
    if out.dtype != torch.bfloat16 or not torch.allclose(out.float(), ref, rtol=0.01, atol=0.01):
        raise RuntimeError("packed W4A8 numerical self-test failed")
    for hidden in (256, 8192):
        x = (((torch.arange(3 * hidden, device=device) % 29) - 14).reshape(3, hidden).to(torch.bfloat16) / 16)
        y = convrot_w4a4_linear(x, torch.zeros((5, hidden // 2), dtype=torch.int8, device=device),
                                torch.ones((5,), dtype=torch.float32, device=device), linear_dtype="int8")
        if y.dtype != torch.bfloat16 or not torch.isfinite(y).all():
            raise RuntimeError(f"BF16 ConvRot W4A8 self-test failed for K={hidden}")
    y = convrot_w4a4_linear(torch.zeros((3, 512), dtype=torch.bfloat16, device=device),
                            torch.zeros((5, 128), dtype=torch.int8, device=device),
                            torch.ones((5,), dtype=torch.float32, device=device), linear_dtype="int8",
                            input_act="swiglu")
    if y.dtype != torch.bfloat16 or not torch.isfinite(y).all():
        raise RuntimeError("SwiGLU W4A8 BF16 self-test failed")
    torch.cuda.synchronize(device)
    _PREFLIGHTED_DEVICES.add(index)


def preflight_codebook_w4a8(device: torch.device) -> None:
    """dispatch.py:153-199: once per device, a numerical self-test of grouped-codebook W4A8
    against a float decode + matmul (the reference's tolerances)."""
    if not is_supported_b200_device(device):
        raise RuntimeError(f"unsupported device {device}")
    if not hasattr(_C, "turing_codebook_w4a8_linear"):
        raise RuntimeError("the installed comfyui-turing-utils-kernel does not provide codebook W4A8")
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index in _PREFLIGHTED_CODEBOOK_DEVICES:
        return
    m, n, k, g = 3, 8, 64, 16
    activation = ((torch.arange(m * k, device=device) % 23) - 11).to(torch.int8).reshape(m, k)
    codes = (torch.arange(n * k, device=device) % 16).to(torch.int32).reshape(n, k)
    packed = ((codes[:, 0::2] & 0x0F) | ((codes[:, 1::2] & 0x0F) << 4)).to(torch.int8)
    codebook = torch.linspace(-0.95, 0.95, 16, dtype=torch.float32, device=device)
    group_scale = torch.linspace(8.0, 32.0, n * (k // g), dtype=torch.float32, device=device).reshape(
        n, k // g).to(torch.float8_e4m3fn)
    c_s = torch.linspace(0.01, 0.03, n, dtype=torch.float32, device=device)
    a_s = torch.linspace(0.02, 0.04, m, dtype=torch.float32, device=device)
    bias = torch.linspace(-0.1, 0.1, n, dtype=torch.bfloat16, device=device)
    out = ops.turing_codebook_w4a8_linear(activation, packed, a_s, group_scale, c_s, codebook, bias, g)
    decoded = (codebook[codes] * group_scale.float().repeat_interleave(g, dim=1)).round().clamp(-127, 127)
    ref = (activation.float() @ decoded.float().t()) * a_s[:, None] * c_s[None, :] + bias.float()
    if out.dtype is not torch.bfloat16 or not torch.allclose(out.float(), ref, rtol=0.01, atol=0.02):
        raise RuntimeError("codebook W4A8 numerical self-test failed")
    _PREFLIGHTED_CODEBOOK_DEVICES.add(index)

