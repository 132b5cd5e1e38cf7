"""B200 (sm_100a) drop-in for the ``comfyui_turing_utils_kernel`` package.

Exports the ConvRot quantized-linear operations of the reference kernel package
(kernel/comfyui_turing_utils_kernel/__init__.py:1-39) implemented by hand-written
tcgen05/TMA CUDA kernels in libctu_b200.so, and the two norm + AdaLN ops that feed
them.  Attention (``turing_sage``) is outside this build's scope.
"""

from .ops import (
    turing_asym_w4a8_g128_linear,
    turing_bf16_gelu_int4_convrot_quantize,
    turing_bf16_gelu_int8_convrot_quantize,
    turing_bf16_int4_convrot_quantize,
    turing_bf16_int4_g128_convrot_quantize,
    turing_bf16_int8_convrot_quantize,
    turing_bf16_int8_convrot_quantize_b128,
    turing_codebook_w4a8_linear,
    turing_convrot_int8_linear,
    turing_dequantize_int8_bf16,
    turing_gelu_int4_convrot_quantize,
    turing_gelu_int8_convrot_quantize,
    turing_int8_linear,
    turing_layer_norm_adaln,
    turing_segmented_rms_adaln,
    turing_swiglu_int4_convrot_quantize,
    turing_swiglu_int8_convrot_quantize,
    turing_swiglu_int8_convrot_quantize_scaled,
    turing_w4a4_g128_linear,
    turing_w4a8_linear,
)

# Version contract checked by the plugin (precision.py:31-32,91-104 of the reference).
__version__ = "0.31.0"
__b200_build__ = "0.1.0"

__all__ = [
    "turing_asym_w4a8_g128_linear",
    "turing_bf16_gelu_int4_convrot_quantize",
    "turing_bf16_gelu_int8_convrot_quantize",
    "turing_bf16_int4_convrot_quantize",
    "turing_bf16_int4_g128_convrot_quantize",
    "turing_bf16_int8_convrot_quantize",
    "turing_bf16_int8_convrot_quantize_b128",
    "turing_codebook_w4a8_linear",
    "turing_convrot_int8_linear",
    "turing_dequantize_int8_bf16",
    "turing_gelu_int4_convrot_quantize",
    "turing_gelu_int8_convrot_quantize",
    "turing_int8_linear",
    "turing_layer_norm_adaln",
    "turing_segmented_rms_adaln",
    "turing_swiglu_int4_convrot_quantize",
    "turing_swiglu_int8_convrot_quantize",
    "turing_swiglu_int8_convrot_quantize_scaled",
    "turing_w4a4_g128_linear",
    "turing_w4a8_linear",
]
