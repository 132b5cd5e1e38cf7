"""Weight-format classification and output-channel slicing of the ConvRot linear.

Mirrors the format-level helpers of the reference plugin
(comfyui_turing_utils/quantization/fusions.py:14-85): the same layout names and
parameter checks decide which B200 kernel a ComfyUI ``QuantizedTensor`` weight maps
to, and ``convrot_w8_output_slice`` evaluates a contiguous interval of output
channels from an activation quantized once.  The segmented RMSNorm + AdaLN wrapper
(fusions.py:198-269) validates and caches the token-to-modulation segment table the
norm kernel takes.  The helpers read only attributes
(``_layout_cls`` and ``_params``), so they work on ComfyUI's tensors without
importing ComfyUI.
"""

from __future__ import annotations

import functools
import operator

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


def normalized_segments(segments, rows: int, parameter_rows: int) -> tuple[int, ...]:
    """fusions.py:198-222: validate (start, stop, modulation_row) triples that must cover
    rows 0..rows-1 contiguously with rows inside the scale/shift table; return them flat."""
    if rows <= 0 or parameter_rows <= 0:
        raise ValueError("segmented RMSNorm+AdaLN dimensions must be positive")
    flat: list[int] = []
    cursor = 0
    for segment in segments:
        if len(segment) != 3:
            raise ValueError("each modulation segment must contain start, stop, and row")
        try:
            start, stop, modulation_row = (operator.index(value) for value in segment)
        except TypeError as exc:
            raise ValueError("modulation segment values must be integers") from exc
        if start != cursor or stop <= start:
            raise ValueError("modulation segments must cover the input contiguously")
        if modulation_row < 0 or modulation_row >= parameter_rows:
            raise ValueError("modulation segment row is outside the scale/shift table")
        flat.extend((start, stop, modulation_row))
        cursor = stop
    if cursor != rows:
        raise ValueError("modulation segments must cover every input row")
    return tuple(flat)


@functools.lru_cache(maxsize=32)
def _cached_segment_table(flat: tuple[int, ...], device_index: int) -> torch.Tensor:
    # fusions.py:225-227: one int32 [S, 3] device table per distinct segmentation.
    return torch.tensor(flat, dtype=torch.int32, device=torch.device("cuda", device_index)).view(-1, 3)


def segment_table(segments, rows: int, parameter_rows: int, device: torch.device) -> torch.Tensor:
    """fusions.py:230-238: the validated, cached device table of ``segments``."""
    flat = normalized_segments(segments, rows, parameter_rows)
    index = device.index if device.index is not None else torch.cuda.current_device()
    return _cached_segment_table(flat, index)


def segmented_rms_adaln(norm, x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, segments) -> torch.Tensor:
    """fusions.py:241-269 without ComfyUI's weight casting: the affine RMSNorm ``norm``
    (its ``weight`` -- ones when None -- and ``eps``; a bias is rejected) followed by
    the segmented AdaLN modulation, on the B200 norm kernel."""
    import comfyui_turing_utils_kernel as ops

    weight = getattr(norm, "weight", None)
    if getattr(norm, "bias", None) is not None:
        raise RuntimeError("segmented RMSNorm+AdaLN does not support a biased norm")
    if weight is None:
        weight = torch.ones(x.shape[-1], dtype=x.dtype, device=x.device)
    weight = weight.to(device=x.device, dtype=x.dtype)
    scale = scale.to(device=x.device, dtype=x.dtype)
    shift = shift.to(device=x.device, dtype=x.dtype)
    table = segment_table(segments, x.shape[0], scale.shape[0], x.device)
    return ops.turing_segmented_rms_adaln(x, weight, scale, shift, table, float(norm.eps))
