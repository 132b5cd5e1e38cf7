"""Kitchen-free mirror of the plugin's ConvRot linear entry points on B200 (see dispatch.py)."""

from .dispatch import (
    convrot_w4a4_linear,
    int8_linear,
    int8_linear_from_quantized,
    quantize_convrot_int8_activation,
    quantize_convrot_swiglu_activation,
)

__all__ = [
    "convrot_w4a4_linear",
    "int8_linear",
    "int8_linear_from_quantized",
    "quantize_convrot_int8_activation",
    "quantize_convrot_swiglu_activation",
]
