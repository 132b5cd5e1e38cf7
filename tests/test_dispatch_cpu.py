"""Argument handling of the kitchen-free dispatch mirror (no GPU needed)."""

import pytest
import torch


def test_unsupported_configurations_raise_not_implemented():
    import comfyui_turing_utils_b200 as d

    x = torch.zeros((2, 256), dtype=torch.float16)
    w = torch.zeros((8, 256), dtype=torch.int8)
    s = torch.ones(8)
    with pytest.raises(NotImplementedError, match="non-bf16"):
        d.int8_linear(x, w, s, convrot=True)
    xb = x.to(torch.bfloat16)
    with pytest.raises(NotImplementedError, match="without ConvRot"):
        d.int8_linear(xb, w, s, convrot=False)
    with pytest.raises(NotImplementedError, match="group size 128"):
        d.int8_linear(xb, w, s, convrot=True, convrot_groupsize=128)
    with pytest.raises(NotImplementedError, match="quant_group_size"):
        d.convrot_w4a4_linear(xb, w, s, quant_group_size=32)


def test_quantize_helpers_validate_inputs():
    import comfyui_turing_utils_b200 as d

    with pytest.raises(ValueError, match="two-dimensional"):
        d.quantize_convrot_int8_activation(torch.zeros((2, 2, 256), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="BF16"):
        d.quantize_convrot_int8_activation(torch.zeros((2, 256)))
    with pytest.raises(ValueError, match="on CUDA"):
        d.quantize_convrot_int8_activation(torch.zeros((2, 256), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match=r"\[M, 2K\]"):
        d.quantize_convrot_swiglu_activation(torch.zeros((2, 255), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="widths differ"):
        d.int8_linear_from_quantized(torch.zeros((2, 256), dtype=torch.int8), torch.ones(2),
                                     torch.zeros((8, 128), dtype=torch.int8), torch.ones(8))
