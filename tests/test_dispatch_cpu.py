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


class _Params:
    def __init__(self, **kw):
        self.orig_dtype = torch.bfloat16
        self.convrot_groupsize = 256
        self.__dict__.update(kw)


class _Weight:
    def __init__(self, layout, **params):
        self._layout_cls = layout
        self._params = _Params(**params)


def test_convrot_weight_kind_follows_the_reference_rules():
    # fusions.py:19-38, one case per rule.
    from comfyui_turing_utils_b200 import convrot_weight_kind, is_turing_convrot_linear

    assert convrot_weight_kind(_Weight("TensorWiseINT8Layout", convrot=True)) == "w8a8"
    assert convrot_weight_kind(_Weight("TensorWiseINT8Layout", convrot=False)) is None
    assert convrot_weight_kind(_Weight("TensorWiseINT8Layout", convrot=True, orig_dtype=torch.float16)) is None
    assert convrot_weight_kind(_Weight("TensorWiseINT8Layout", convrot=True, transposed=True)) is None
    assert convrot_weight_kind(_Weight("TensorWiseINT8Layout", convrot=True, convrot_groupsize=128)) is None
    w4 = "TensorCoreConvRotW4A4Layout"
    assert convrot_weight_kind(_Weight(w4, quant_group_size=64, linear_dtype="int4")) == "w4a4"
    assert convrot_weight_kind(_Weight(w4, quant_group_size=64, linear_dtype="int8")) == "w4a8"
    assert convrot_weight_kind(_Weight(w4, quant_group_size=64, linear_dtype="fp8")) is None
    assert convrot_weight_kind(_Weight(w4, quant_group_size=32, linear_dtype="int4")) is None
    cb = "AsymW4A8Int8Layout"
    assert convrot_weight_kind(_Weight(cb, group_size=16, codebook=torch.zeros(16), correction=None)) == "codebook_w4a8"
    assert convrot_weight_kind(_Weight(cb, group_size=2, codebook=torch.zeros(16), correction=None)) is None
    assert convrot_weight_kind(_Weight(cb, group_size=16, codebook=None, correction=None)) is None
    assert convrot_weight_kind(_Weight(cb, group_size=16, codebook=torch.zeros(16), correction=torch.zeros(1))) is None
    assert convrot_weight_kind(None) is None
    linear = torch.nn.Module()
    linear.weight = _Weight("TensorWiseINT8Layout", convrot=True)
    assert is_turing_convrot_linear(linear)


def test_w8_output_slice_rejects_out_of_range_intervals():
    from comfyui_turing_utils_b200 import convrot_w8_output_slice

    q = torch.zeros((2, 256), dtype=torch.int8)
    w = torch.zeros((8, 256), dtype=torch.int8)
    for start, stop in ((-1, 4), (4, 4), (0, 9)):
        with pytest.raises(ValueError, match="outside the weight"):
            convrot_w8_output_slice(q, torch.ones(2), w, torch.ones(8), None, start, stop, torch.bfloat16)
