"""Weight-format classification and output-channel slicing of the ConvRot linear.

Mirrors the format-level helpers of the reference plugin
(comfyui_turing_utils/quantization/fusions.py:14-85): the same layout names and
parameter checks decide which B200 kernel a ComfyUI ``QuantizedTensor`` weight maps
to, and ``convrot_w8_output_slice`` evaluates a contiguous interval of output
channels from an activation quantized once.  The helpers read only attributes
(``_layout_cls`` and ``_params``), so they work on ComfyUI's tensors without
importing ComfyUI.
"""

from __future__ import annotations

import torch

from .dispatch import int8_linear_from_quantized

W8_LAYOUT = "TensorWiseINT8Layout"
W4_LAYOUT = "TensorCoreConvRotW4A4Layout"
CODEBOOK_W4_LAYOUT = "AsymW4A8Int8Layout"


def convrot_weight_kind(weight) -> str | None:
    """fusions.py:19-38: ``"w8a8"``, ``"w4a8"``, ``"w4a4"``, ``"codebook_w4a8"`` or None.

    A weight qualifies only when it was quantized from bf16, is not transposed and
    uses ConvRot group 256; W4 additionally needs ``quant_group_size == 64`` and an
    int4/int8 ``linear_dtype``; the grouped codebook needs ``group_size >= 4``, a
    codebook and no correction term.
    """
    params = getattr(weight, "_params", None)
    if getattr(params, "orig_dtype", None) is not torch.bfloat16:
        return None
    if getattr(params, "transposed", False) or getattr(params, "convrot_groupsize", None) != 256:
        return None
    layout = getattr(weight, "_layout_cls", None)
    if layout == W8_LAYOUT and getattr(params, "convrot", False):
        return "w8a8"
    if layout == W4_LAYOUT and getattr(params, "quant_group_size", None) == 64:
        linear_dtype = getattr(params, "linear_dtype", None)
        return f"w4a{linear_dtype[-1]}" if linear_dtype in {"int4", "int8"} else None
    group_size = getattr(params, "group_size", None)
    if (
        layout == CODEBOOK_W4_LAYOUT
        and isinstance(group_size, int)
        and group_size >= 4
        and getattr(params, "codebook", None) is not None
        and getattr(params, "correction", None) is None
    ):
        return "codebook_w4a8"
    return None


def is_turing_convrot_linear(linear: torch.nn.Module) -> bool:
    """fusions.py:41-42."""
    return convrot_weight_kind(getattr(linear, "weight", None)) is not None


def convrot_w8_output_slice(
    qactivation: torch.Tensor,
    activation_scale: torch.Tensor,
    qweight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None,
    start: int,
    stop: int,
    output_dtype: torch.dtype,
) -> torch.Tensor:
    """fusions.py:56-85: the W8 linear restricted to output channels [start, stop)."""
    start, stop = int(start), int(stop)
    if start < 0 or stop <= start or stop > qweight.shape[0]:
        raise ValueError("W8 output slice is outside the weight")
    sliced_scale = weight_scale if weight_scale.numel() == 1 else weight_scale.reshape(-1)[start:stop]
    sliced_bias = None if bias is None else bias[start:stop]
    return int8_linear_from_quantized(
        qactivation,
        activation_scale,
        qweight[start:stop],
        sliced_scale,
        bias=sliced_bias,
        out_dtype=output_dtype,
    )
