"""``turing_utils::*`` torch custom ops over the B200 kernels.

Op names, signatures, defaults, device/capability errors and fake (meta) kernels
follow the reference's kernel/comfyui_turing_utils_kernel/ops.py, so graph capture,
torch.compile tracing and shape propagation see the same contract.  Each op calls
the matching function of ``_C`` (the C-ABI shim); there is no CPU path.
"""

from __future__ import annotations

import torch

from . import _C


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{what} requires CUDA tensors")
    if torch.cuda.get_device_capability(t.device) < (7, 5):
        raise RuntimeError(f"{what} requires sm75 or newer")


# ops.py:8-35
@torch.library.custom_op("turing_utils::w4a8_linear", mutates_args=())
def turing_w4a8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Signed packed-int4 W4A8 linear (int4 sign-extended in shared memory, tcgen05 MMA)."""
    _require_cuda(activation, "Turing W4A8")
    return _C.turing_w4a8_linear(
        activation.contiguous(),
        weight.contiguous(),
        activation_scale.contiguous(),
        weight_scale.contiguous(),
        None if bias is None else bias.contiguous(),
    )


@turing_w4a8_linear.register_fake
def _turing_w4a8_linear_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16, device=activation.device)


# ops.py:38-93
@torch.library.custom_op("turing_utils::codebook_w4a8_linear", mutates_args=())
def turing_codebook_w4a8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    group_scale: torch.Tensor,
    channel_scale: torch.Tensor,
    codebook: torch.Tensor,
    bias: torch.Tensor | None = None,
    group_size: int = 16,
    chunk_rows: int = 0,
) -> torch.Tensor:
    """Grouped-codebook W4A8: codes decoded to int8 ahead of the tcgen05 GEMM.

    ``chunk_rows=0`` selects the production policy, ``-1`` forces the long-sequence
    policy (group_size 16, M > 8192), and a positive multiple of eight forces that many
    output channels per decoded chunk.
    """
    _require_cuda(activation, "Turing codebook W4A8")
    if group_scale.dtype == torch.float8_e4m3fn:
        group_scale = group_scale.view(torch.uint8)
    if group_scale.dtype != torch.uint8:
        raise TypeError("group_scale must be float8_e4m3fn or its raw uint8 view")
    return _C.turing_codebook_w4a8_linear(
        activation.contiguous(), weight.contiguous(), activation_scale.contiguous(), group_scale.contiguous(),
        channel_scale.contiguous(), codebook.contiguous(), None if bias is None else bias.contiguous(),
        group_size, chunk_rows)


@turing_codebook_w4a8_linear.register_fake
def _turing_codebook_w4a8_linear_fake(activation, weight, activation_scale, group_scale, channel_scale, codebook,
                                      bias=None, group_size=16, chunk_rows=0):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16, device=activation.device)


@torch.library.custom_op("turing_utils::int8_linear", mutates_args=())
def turing_int8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """W8A8 contraction with the fused dequant + bias epilogue (tcgen05 kind::i8)."""
    _require_cuda(activation, "Turing INT8 linear")
    return _C.turing_int8_linear(
        activation.contiguous(),
        weight.contiguous(),
        activation_scale.contiguous(),
        weight_scale.contiguous(),
        None if bias is None else bias.contiguous(),
    )


@turing_int8_linear.register_fake
def _turing_int8_linear_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16, device=activation.device)


@torch.library.custom_op("turing_utils::bf16_int8_convrot_quantize_b128", mutates_args=())
def turing_bf16_int8_convrot_quantize_b128(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """ConvRot int8 quantize with rotation block 128 (no reference op: the reference's
    quantizers take block 256 only; the block-128 rotation is defined in ctu_b200.h)."""
    _require_cuda(x, "block-128 ConvRot")
    return _C.bf16_int8_convrot_quantize_b128(x.contiguous())


@turing_bf16_int8_convrot_quantize_b128.register_fake
def _turing_bf16_int8_convrot_quantize_b128_fake(x):
    return (torch.empty_like(x, dtype=torch.int8),
            torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))


@torch.library.custom_op("turing_utils::convrot_int8_linear", mutates_args=())
def turing_convrot_int8_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    group_size: int = 256,
) -> torch.Tensor:
    """ConvRot W8A8 linear from bf16 rows (quantize + int8_linear in one call; no
    reference op: the plugin composes the two in dispatch.int8_linear, dispatch.py:748-800)."""
    _require_cuda(x, "ConvRot INT8 linear")
    return _C.convrot_int8_linear(x, weight, weight_scale, bias, group_size)


@turing_convrot_int8_linear.register_fake
def _turing_convrot_int8_linear_fake(x, weight, weight_scale, bias=None, group_size=256):
    return torch.empty((x.size(0), weight.size(0)), dtype=torch.bfloat16, device=x.device)


# ops.py:129-160
@torch.library.custom_op("turing_utils::dequantize_int8_bf16", mutates_args=())
def turing_dequantize_int8_bf16(
    accumulator: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    output_columns: int = -1,
) -> torch.Tensor:
    """Dequantize an INT32 GEMM workspace directly into bf16."""
    _require_cuda(accumulator, "Turing BF16 epilogue")
    if accumulator.dtype != torch.int32 or accumulator.ndim != 2:
        raise TypeError("accumulator must be a 2D int32 tensor")
    return _C.turing_dequantize_int8_bf16(
        accumulator.contiguous(), activation_scale.contiguous(), weight_scale.contiguous(), output_columns
    )


@turing_dequantize_int8_bf16.register_fake
def _turing_dequantize_int8_bf16_fake(accumulator, activation_scale, weight_scale, output_columns=-1):
    columns = accumulator.size(1) if output_columns < 0 else output_columns
    return torch.empty((accumulator.size(0), columns), dtype=torch.bfloat16, device=accumulator.device)


def _check_bf16_2d(x: torch.Tensor, what: str) -> None:
    if x.dtype != torch.bfloat16:
        raise TypeError(f"{what} input must be bfloat16")
    if x.ndim != 2:
        raise ValueError(f"{what} input must be 2D")


# ops.py:290-315
@torch.library.custom_op("turing_utils::bf16_int8_convrot_quantize", mutates_args=())
def turing_bf16_int8_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
    *,
    swiglu: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused ConvRot rotation + per-token int8 quantization of a bf16 row block."""
    _require_cuda(x, "BF16 row-buffer ConvRot")
    _check_bf16_2d(x, "BF16 row-buffer ConvRot")
    return _C.turing_bf16_int8_convrot_quantize(x.contiguous(), group_size, swiglu)


@turing_bf16_int8_convrot_quantize.register_fake
def _turing_bf16_int8_convrot_quantize_fake(x, group_size=256, *, swiglu=False):
    hidden = x.size(1) // 2 if swiglu else x.size(1)
    return (
        torch.empty((x.size(0), hidden), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:318-343
@torch.library.custom_op("turing_utils::bf16_int4_convrot_quantize", mutates_args=())
def turing_bf16_int4_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
    *,
    swiglu: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused ConvRot rotation + per-token packed-int4 quantization."""
    _require_cuda(x, "BF16 row-buffer INT4 ConvRot")
    _check_bf16_2d(x, "BF16 row-buffer INT4 ConvRot")
    return _C.turing_bf16_int4_convrot_quantize(x.contiguous(), group_size, swiglu)


@turing_bf16_int4_convrot_quantize.register_fake
def _turing_bf16_int4_convrot_quantize_fake(x, group_size=256, *, swiglu=False):
    hidden = x.size(1) // 2 if swiglu else x.size(1)
    return (
        torch.empty((x.size(0), hidden // 2), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:346-365
@torch.library.custom_op("turing_utils::bf16_gelu_int8_convrot_quantize", mutates_args=())
def turing_bf16_gelu_int8_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused tanh-GELU + ConvRot + per-token int8 quantization."""
    _require_cuda(x, "BF16 GELU ConvRot")
    _check_bf16_2d(x, "BF16 GELU ConvRot")
    return _C.turing_bf16_gelu_int8_convrot_quantize(x.contiguous(), group_size)


@turing_bf16_gelu_int8_convrot_quantize.register_fake
def _turing_bf16_gelu_int8_convrot_quantize_fake(x, group_size=256):
    return (
        torch.empty(x.shape, dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:368-385
@torch.library.custom_op("turing_utils::bf16_gelu_int4_convrot_quantize", mutates_args=())
def turing_bf16_gelu_int4_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused tanh-GELU + ConvRot + per-token packed-int4 quantization."""
    _require_cuda(x, "BF16 GELU INT4 ConvRot")
    _check_bf16_2d(x, "BF16 GELU INT4 ConvRot")
    return _C.turing_bf16_gelu_int4_convrot_quantize(x.contiguous(), group_size)


@turing_bf16_gelu_int4_convrot_quantize.register_fake
def _turing_bf16_gelu_int4_convrot_quantize_fake(x, group_size=256):
    return (
        torch.empty((x.size(0), x.size(1) // 2), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:163-186, 222-287: the staged entries share the fused kernel (bf16 input).
@torch.library.custom_op("turing_utils::swiglu_int8_convrot_quantize", mutates_args=())
def turing_swiglu_int8_convrot_quantize(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """SwiGLU + ConvRot int8 quantization of a [M, 2K] (gate | up) block."""
    _require_cuda(x, "Turing SwiGLU ConvRot")
    if x.ndim != 2:
        raise ValueError("SwiGLU ConvRot input must be 2D [M, 2K]")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("SwiGLU ConvRot input must be float16 or bfloat16")
    return _C.turing_swiglu_int8_convrot_quantize(x.contiguous(), group_size)


@turing_swiglu_int8_convrot_quantize.register_fake
def _turing_swiglu_int8_convrot_quantize_fake(x, group_size=256):
    hidden = x.size(1) // 2
    return (
        torch.empty((x.size(0), hidden), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:189-219: one channel shard quantized with precomputed whole-row scales.
@torch.library.custom_op("turing_utils::swiglu_int8_convrot_quantize_scaled", mutates_args=())
def turing_swiglu_int8_convrot_quantize_scaled(
    x: torch.Tensor,
    scales: torch.Tensor,
    group_size: int = 256,
) -> torch.Tensor:
    """Quantize a SwiGLU+ConvRot shard with precomputed whole-row scales."""
    _require_cuda(x, "scaled Turing SwiGLU ConvRot")
    if x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2:
        raise TypeError("scaled SwiGLU ConvRot input must be 2D float16 or bfloat16")
    if scales.dtype != torch.float32 or scales.numel() != x.shape[0]:
        raise TypeError("scaled SwiGLU ConvRot requires one FP32 scale per row")
    return _C.turing_swiglu_int8_convrot_quantize_scaled(x.contiguous(), scales.contiguous(), group_size)


@turing_swiglu_int8_convrot_quantize_scaled.register_fake
def _turing_swiglu_int8_convrot_quantize_scaled_fake(x, scales, group_size=256):
    return torch.empty((x.size(0), x.size(1) // 2), dtype=torch.int8, device=x.device)


@torch.library.custom_op("turing_utils::swiglu_int4_convrot_quantize", mutates_args=())
def turing_swiglu_int4_convrot_quantize(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """SwiGLU + ConvRot packed-int4 quantization of a [M, 2K] block."""
    _require_cuda(x, "Turing SwiGLU INT4 ConvRot")
    if x.ndim != 2:
        raise ValueError("SwiGLU INT4 ConvRot input must be 2D [M, 2K]")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("SwiGLU INT4 ConvRot input must be float16 or bfloat16")
    return _C.turing_swiglu_int4_convrot_quantize(x.contiguous(), group_size)


@turing_swiglu_int4_convrot_quantize.register_fake
def _turing_swiglu_int4_convrot_quantize_fake(x, group_size=256):
    hidden = x.size(1) // 2
    return (
        torch.empty((x.size(0), hidden // 2), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


@torch.library.custom_op("turing_utils::gelu_int8_convrot_quantize", mutates_args=())
def turing_gelu_int8_convrot_quantize(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """tanh-GELU + ConvRot int8 quantization."""
    _require_cuda(x, "Turing GELU ConvRot")
    if x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2:
        raise TypeError("GELU ConvRot input must be 2D float16 or bfloat16")
    return _C.turing_gelu_int8_convrot_quantize(x.contiguous(), group_size)


@turing_gelu_int8_convrot_quantize.register_fake
def _turing_gelu_int8_convrot_quantize_fake(x, group_size=256):
    return (
        torch.empty(x.shape, dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


@torch.library.custom_op("turing_utils::gelu_int4_convrot_quantize", mutates_args=())
def turing_gelu_int4_convrot_quantize(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """tanh-GELU + ConvRot packed-int4 quantization."""
    _require_cuda(x, "Turing GELU INT4 ConvRot")
    if x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2:
        raise TypeError("GELU INT4 ConvRot input must be 2D float16 or bfloat16")
    return _C.turing_gelu_int4_convrot_quantize(x.contiguous(), group_size)


@turing_gelu_int4_convrot_quantize.register_fake
def _turing_gelu_int4_convrot_quantize_fake(x, group_size=256):
    return (
        torch.empty((x.size(0), x.size(1) // 2), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device),
    )


# ops.py:388-425
@torch.library.custom_op("turing_utils::segmented_rms_adaln", mutates_args=())
def turing_segmented_rms_adaln(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    segments: torch.Tensor,
    epsilon: float = 1.0e-5,
) -> torch.Tensor:
    """Fused affine RMSNorm and segmented AdaLN modulation."""
    if x.device.type != "cuda":
        raise RuntimeError("Segmented RMSNorm+AdaLN requires CUDA tensors")
    if torch.cuda.get_device_capability(x.device) < (7, 5):
        raise RuntimeError("Segmented RMSNorm+AdaLN requires sm75 or newer")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("segmented RMSNorm+AdaLN input must be float16, bfloat16, or float32")
    if x.ndim != 2:
        raise ValueError("segmented RMSNorm+AdaLN input must be 2D [M, K]")
    if weight.device != x.device or scale.device != x.device or shift.device != x.device:
        raise ValueError("weight, scale, and shift must be on the input device")
    weight = weight.to(dtype=x.dtype).contiguous()
    scale = scale.to(dtype=x.dtype)
    shift = shift.to(dtype=x.dtype)
    if scale.stride(-1) != 1:
        scale = scale.contiguous()
    if shift.stride(-1) != 1:
        shift = shift.contiguous()
    if segments.device != x.device or segments.dtype != torch.int32:
        raise ValueError("segments must be an int32 tensor on the input device")
    return _C.turing_segmented_rms_adaln(x.contiguous(), weight, scale, shift, segments.contiguous(), epsilon)


@turing_segmented_rms_adaln.register_fake
def _turing_segmented_rms_adaln_fake(x, weight, scale, shift, segments, epsilon=1.0e-5):
    return torch.empty_like(x)


# ops.py:432-447
@torch.library.custom_op("turing_utils::layer_norm_adaln", mutates_args=())
def turing_layer_norm_adaln(
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    epsilon: float = 1.0e-5,
) -> torch.Tensor:
    """Fused FP32-reduction LayerNorm and Wan AdaLN modulation."""
    if x.device.type != "cuda" or torch.cuda.get_device_capability(x.device) < (7, 5):
        raise RuntimeError("LayerNorm+AdaLN requires an sm75-or-newer CUDA tensor")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32) or x.ndim != 3:
        raise TypeError("LayerNorm+AdaLN input must be 3D float16, bfloat16, or float32")
    scale = scale.to(device=x.device, dtype=x.dtype).contiguous()
    shift = shift.to(device=x.device, dtype=x.dtype).contiguous()
    return _C.turing_layer_norm_adaln(x.contiguous(), scale, shift, epsilon)


@turing_layer_norm_adaln.register_fake
def _turing_layer_norm_adaln_fake(x, scale, shift, epsilon=1.0e-5):
    return torch.empty_like(x)


# Per-group (128 along K) formats.  No reference op carries them (the reference's W4A4
# path calls comfy-kitchen's int4_linear with 64-column weight groups, dispatch.py:876-936,
# and it has no per-group asymmetric W4A8 format); the names follow the turing_utils::
# convention and the arithmetic is documented in ctu_b200.h.
@torch.library.custom_op("turing_utils::bf16_int4_g128_convrot_quantize", mutates_args=())
def turing_bf16_int4_g128_convrot_quantize(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """ConvRot rotation + int4 codes with one scale per token per 128 columns."""
    _require_cuda(x, "per-group INT4 ConvRot")
    _check_bf16_2d(x, "per-group INT4 ConvRot")
    return _C.bf16_int4_g128_convrot_quantize(x.contiguous(), group_size)


@turing_bf16_int4_g128_convrot_quantize.register_fake
def _turing_bf16_int4_g128_convrot_quantize_fake(x, group_size=256):
    return (
        torch.empty((x.size(0), x.size(1) // 2), dtype=torch.int8, device=x.device),
        torch.empty((x.size(0), x.size(1) // 128), dtype=torch.float32, device=x.device),
    )


@torch.library.custom_op("turing_utils::asym_w4a8_g128_linear", mutates_args=())
def turing_asym_w4a8_g128_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    weight_zero: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Asymmetric uint4 W4A8: fp16 scale and uint4 zero point per 128 columns of K."""
    _require_cuda(activation, "asymmetric W4A8")
    return _C.asym_w4a8_g128_linear(activation, weight, activation_scale, weight_scale, weight_zero, bias)


@turing_asym_w4a8_g128_linear.register_fake
def _turing_asym_w4a8_g128_linear_fake(activation, weight, activation_scale, weight_scale, weight_zero, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16, device=activation.device)


@torch.library.custom_op("turing_utils::w4a4_g128_linear", mutates_args=())
def turing_w4a4_g128_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """W4A4 with per-token-per-group-128 activation scales and fp16 per-group weight scales."""
    _require_cuda(activation, "per-group W4A4")
    return _C.w4a4_g128_linear(activation, weight, activation_scale, weight_scale, bias)


@turing_w4a4_g128_linear.register_fake
def _turing_w4a4_g128_linear_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16, device=activation.device)
