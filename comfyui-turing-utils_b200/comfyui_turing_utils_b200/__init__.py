"""Kitchen-free mirror of the plugin's ConvRot linear entry points on B200 (see dispatch.py
and fusions.py)."""

from .dispatch import (
    codebook_w4a8_linear,
    convrot_swiglu_channel_sharding_available,
    convrot_w4a4_linear,
    int8_linear,
    int8_linear_from_quantized,
    preflight_codebook_w4a8,
    preflight_w4a8,
    quantize_convrot_int8_activation,
    quantize_convrot_swiglu_activation,
    quantize_convrot_swiglu_with_scale,
    turing_codebook_w4a8_workspace_bytes,
    turing_int8_workspace_bytes,
    w4a8_int8_linear,
)
from .fusions import (
    convrot_w8_output_slice,
    convrot_weight_kind,
    is_turing_convrot_linear,
    normalized_segments,
    segment_table,
    segmented_rms_adaln,
)

__all__ = [
    "codebook_w4a8_linear",
    "convrot_swiglu_channel_sharding_available",
    "convrot_w4a4_linear",
    "convrot_w8_output_slice",
    "convrot_weight_kind",
    "int8_linear",
    "int8_linear_from_quantized",
    "is_turing_convrot_linear",
    "normalized_segments",
    "segment_table",
    "segmented_rms_adaln",
    "preflight_codebook_w4a8",
    "preflight_w4a8",
    "quantize_convrot_int8_activation",
    "quantize_convrot_swiglu_activation",
    "quantize_convrot_swiglu_with_scale",
    "turing_codebook_w4a8_workspace_bytes",
    "turing_int8_workspace_bytes",
    "w4a8_int8_linear",
]
