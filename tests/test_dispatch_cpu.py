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


def test_workspace_helpers_report_the_b200_workspaces():
    import comfyui_turing_utils_b200 as d

    # The W8A8 GEMM never stages int32 accumulators (dispatch.py:32-43 returns the
    # reference's M*N*4 staging size below 64 MiB).
    assert d.turing_int8_workspace_bytes(4096, 5120) == 0
    assert d.turing_int8_workspace_bytes(0, 5120) == 0
    # Grouped W4A8 decodes all channels at once while their int8 weights fit 256 MiB.
    assert d.turing_codebook_w4a8_workspace_bytes(5120, 5120) == 5120 * 5120
    assert d.turing_codebook_w4a8_workspace_bytes(5376, 28672) == 28672 * 5376
    # Above the budget: 8-row-aligned chunks of at most 256 MiB.
    assert d.turing_codebook_w4a8_workspace_bytes(13824, 28672) == (256 * 2**20 // 13824) // 8 * 8 * 13824
    assert d.turing_codebook_w4a8_workspace_bytes(13824, 28672) <= 256 * 2**20
    assert d.turing_codebook_w4a8_workspace_bytes(0, 8) == 0
    from comfyui_turing_utils_b200 import dispatch

    assert dispatch.TURING_CODEBOOK_W4A8_CHUNK_ROWS == 4096


def test_channel_sharding_probe_and_preflight_device_checks():
    import comfyui_turing_utils_b200 as d

    assert d.convrot_swiglu_channel_sharding_available()
    # Without a B200 the preflights refuse the device, as the reference's do for
    # non-Turing devices (dispatch.py:89-90,155-156).
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="unsupported device"):
            d.preflight_w4a8(torch.device("cuda", 0))
        with pytest.raises(RuntimeError, match="unsupported device"):
            d.preflight_codebook_w4a8(torch.device("cuda", 0))
    with pytest.raises(RuntimeError, match="unsupported device"):
        d.preflight_w4a8(torch.device("cpu"))


def test_preflights_report_missing_kernels(monkeypatch):
    # Mirrors tests/test_turing_policy.py:359-373 of the reference: a kernel package
    # without the op fails the preflight with a message naming it.
    import comfyui_turing_utils_b200 as d
    from comfyui_turing_utils_b200 import dispatch

    monkeypatch.setattr(dispatch, "is_supported_b200_device", lambda device: True)
    monkeypatch.delattr(dispatch._C, "turing_w4a8_linear")
    monkeypatch.delattr(dispatch._C, "turing_codebook_w4a8_linear")
    with pytest.raises(RuntimeError, match="does not provide W4A8"):
        d.preflight_w4a8(torch.device("cuda", 0))
    with pytest.raises(RuntimeError, match="codebook W4A8"):
        d.preflight_codebook_w4a8(torch.device("cuda", 0))


def test_segment_validation_follows_the_reference_rules():
    # tests/test_turing_fusions.py:19-33 of the reference.
    from comfyui_turing_utils_b200 import normalized_segments

    assert normalized_segments([(0, 1, 2), (1, 7, 0), (7, 19, 1)], 19, 3) == (0, 1, 2, 1, 7, 0, 7, 19, 1)
    with pytest.raises(ValueError, match="contiguously"):
        normalized_segments([(0, 2, 0), (3, 4, 0)], 4, 1)
    with pytest.raises(ValueError, match="outside"):
        normalized_segments([(0, 4, 1)], 4, 1)
    with pytest.raises(ValueError, match="every input row"):
        normalized_segments([(0, 3, 0)], 4, 1)
    with pytest.raises(ValueError, match="start, stop, and row"):
        normalized_segments([(0, 4)], 4, 1)
    with pytest.raises(ValueError, match="integers"):
        normalized_segments([(0, 4.0, 0)], 4, 1)
    with pytest.raises(ValueError, match="positive"):
        normalized_segments([(0, 4, 0)], 4, 0)


def test_segmented_norm_wrapper_rejects_a_biased_norm():
    from types import SimpleNamespace

    from comfyui_turing_utils_b200 import segmented_rms_adaln

    norm = SimpleNamespace(weight=None, bias=torch.zeros(8), eps=1e-6)
    with pytest.raises(RuntimeError, match="biased norm"):
        segmented_rms_adaln(norm, torch.zeros((2, 8)), torch.zeros((1, 8)), torch.zeros((1, 8)), [(0, 2, 0)])
