"""ConvRot checkpoint metadata (comfyui_turing_utils_b200.checkpoint): the behaviour the
reference's tests/test_convrot_nodes.py:50-327,370-487 require of
configure_convrot_activation and of the model-file filter, restated as tests of the
B200 package (no ComfyUI needed)."""

import json

import pytest
import torch

from comfyui_turing_utils_b200.checkpoint import (
    ConvRotSummary,
    classify_layer,
    configure_convrot_activation,
    convrot_skip_reason,
    decode_quant_tensor,
    encode_quant_tensor,
    kernel_for,
)


def qt(config):
    return encode_quant_tensor(config)


def header(layers):
    return {"_quantization_metadata": json.dumps({"layers": layers})}


def test_codebook_layers_are_counted_and_keep_their_config():
    key = "blocks.0.mlp.fc1.comfy_quant"
    sd = {key: qt({"format": "asym_w4a8_int8", "group_size": 16, "convrot": True, "convrot_groupsize": 256})}
    _, summary = configure_convrot_activation(sd, None, True)
    assert summary == ConvRotSummary(codebook_w4a8=1)
    assert "linear_dtype" not in decode_quant_tensor(sd[key], key)


@pytest.mark.parametrize("config,match", [
    ({"format": "asym_w4a8_int8", "convrot": False}, "must declare convrot=true"),
    ({"format": "asym_w4a8_int8", "group_size": 2}, "invalid group_size"),
    ({"format": "asym_w4a8_int8", "group_size": True}, "invalid group_size"),
    ({"format": "asym_w4a8_int8", "convrot_groupsize": 128}, "requires convrot_groupsize=256"),
    ({"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"}, "INT8 activations only"),
    ({"format": "float8_e4m3fn", "convrot": True}, "unsupported weight format"),
    ({"convrot": True, "convrot_groupsize": 256}, "unsupported weight format None"),
    ({"format": "convrot_w4a4", "linear_dtype": "fp8"}, "unsupported linear_dtype"),
    ({"format": "int8_tensorwise", "convrot": "yes"}, "non-boolean convrot"),
    ({"format": "int8_tensorwise", "params": [1]}, "non-object params"),
])
def test_invalid_layer_configs_are_rejected(config, match):
    with pytest.raises(ValueError, match=match):
        configure_convrot_activation({"blocks.0.ffn.0.comfy_quant": qt(config)}, None, False)


def test_w4_default_is_w4a4_and_header_configs_are_untouched():
    updated, summary = configure_convrot_activation({}, header({"blocks.0.ffn.0": {"format": "convrot_w4a4"}}), False)
    assert summary == ConvRotSummary(w4a4=1)
    assert "linear_dtype" not in json.loads(updated["_quantization_metadata"])["layers"]["blocks.0.ffn.0"]


def test_force_int8_rewrites_header_and_tensor_configs():
    sd = {"blocks.1.ffn.0.comfy_quant": qt({"format": "convrot_w4a4", "linear_dtype": "int4"})}
    updated, summary = configure_convrot_activation(sd, header({"blocks.0.ffn.0": {"format": "convrot_w4a4"}}), True)
    assert json.loads(updated["_quantization_metadata"])["layers"]["blocks.0.ffn.0"]["linear_dtype"] == "int8"
    assert decode_quant_tensor(sd["blocks.1.ffn.0.comfy_quant"], "k")["linear_dtype"] == "int8"
    assert summary == ConvRotSummary(w4a8=2)


def test_model_prefix_limits_which_layers_are_rewritten():
    dit, te = "model.diffusion_model.blocks.0.ffn.0.comfy_quant", "text_encoders.qwen.layers.0.mlp.comfy_quant"
    sd = {dit: qt({"format": "convrot_w4a4", "linear_dtype": "int4"}),
          te: qt({"format": "convrot_w4a4", "linear_dtype": "int4"})}
    _, summary = configure_convrot_activation(sd, None, True, model_prefix="model.diffusion_model.")
    assert summary == ConvRotSummary(w4a8=1)
    assert decode_quant_tensor(sd[dit], dit)["linear_dtype"] == "int8"
    assert decode_quant_tensor(sd[te], te)["linear_dtype"] == "int4"


def test_mixed_w4_and_w8_and_explicit_w4a8():
    sd = {"blocks.0.ffn.0.comfy_quant": qt({"format": "convrot_w4a4"}),
          "blocks.1.ffn.0.comfy_quant": qt({"format": "int8_tensorwise", "params": {"convrot": True}})}
    assert configure_convrot_activation(sd, None, True)[1] == ConvRotSummary(w4a8=1, w8a8=1)
    sd = {"blocks.0.ffn.0.comfy_quant": qt({"format": "convrot_w4a4", "params": {"linear_dtype": "int8"}})}
    assert configure_convrot_activation(sd, None, False)[1] == ConvRotSummary(w4a8=1)


def test_legacy_w8_spellings_are_normalised():
    key = "double_blocks.0.img_attn.qkv.comfy_quant"
    sd = {key: qt({"convrot": True, "convrot_groupsize": 256, "per_row": True})}
    assert configure_convrot_activation(sd, None, False)[1] == ConvRotSummary(w8a8=1)
    assert decode_quant_tensor(sd[key], key)["format"] == "int8_tensorwise"
    legacy = header({"double_blocks.0.img_attn.qkv": {"format": "int8_rowwise", "convrot": True,
                                                      "convrot_groupsize": 256, "per_row": True}})
    updated, summary = configure_convrot_activation({}, legacy, False)
    assert summary == ConvRotSummary(w8a8=1)
    assert json.loads(updated["_quantization_metadata"])["layers"]["double_blocks.0.img_attn.qkv"]["format"] == \
        "int8_tensorwise"


def test_force_int8_accepts_w8_configs_declaring_int4():
    key = "blocks.0.ffn.0.comfy_quant"
    sd = {key: qt({"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"})}
    assert configure_convrot_activation(sd, None, True)[1] == ConvRotSummary(w8a8=1)
    assert decode_quant_tensor(sd[key], key)["linear_dtype"] == "int8"


def test_models_without_convrot_layers_and_malformed_metadata_are_rejected():
    with pytest.raises(ValueError, match="does not contain supported ConvRot"):
        configure_convrot_activation({"a.comfy_quant": qt({"format": "int8_tensorwise"})}, None, False)
    with pytest.raises(ValueError, match="Conflicting ConvRot metadata"):
        configure_convrot_activation({"blocks.0.ffn.0.comfy_quant": qt({"format": "convrot_w4a4"})},
                                     header({"blocks.0.ffn.0": {"format": "convrot_w4a4", "linear_dtype": "int8"}}),
                                     False)
    with pytest.raises(ValueError, match="contains invalid JSON"):
        configure_convrot_activation({}, {"_quantization_metadata": "{"}, False)
    with pytest.raises(ValueError, match="must contain a layers object"):
        configure_convrot_activation({}, {"_quantization_metadata": "[]"}, False)
    with pytest.raises(ValueError, match="contains invalid quantization JSON"):
        configure_convrot_activation({"a.comfy_quant": torch.tensor(list(b"{"), dtype=torch.uint8)}, None, False)
    with pytest.raises(ValueError, match="force_int8_gemm must be boolean"):
        configure_convrot_activation({}, None, "int8")


def test_kernel_for_names_the_dispatch_entry_of_every_kind():
    assert kernel_for(classify_layer({"format": "int8_tensorwise", "convrot": True}, "l", False)) == "int8_linear"
    assert kernel_for(classify_layer({"format": "convrot_w4a4"}, "l", False)).endswith("'int4')")
    assert kernel_for(classify_layer({"format": "convrot_w4a4"}, "l", True)).endswith("'int8')")
    assert kernel_for(classify_layer({"format": "asym_w4a8_int8"}, "l", False)) == "codebook_w4a8_linear"


# ----------------------------------------------------------------------------- model-file filter
def _save(path, tensors, metadata=None):
    from safetensors.torch import save_file

    save_file(tensors, str(path), metadata=metadata)
    return path


def test_files_with_convrot_tensor_or_header_metadata_are_accepted(tmp_path):
    assert convrot_skip_reason(_save(tmp_path / "a.safetensors",
                                     {"blocks.0.ffn.0.comfy_quant": qt({"format": "convrot_w4a4"})})) is None
    assert convrot_skip_reason(_save(tmp_path / "b.safetensors", {"blocks.0.ffn.0.weight": torch.zeros((1, 1))},
                                     header({"blocks.0.ffn.0": {"format": "convrot_w4a4"}}))) is None
    legacy = {"double_blocks.0.img_attn.qkv.comfy_quant": qt({"convrot": True, "convrot_groupsize": 256,
                                                              "per_row": True})}
    assert convrot_skip_reason(_save(tmp_path / "c.sft", legacy)) is None
    text_encoder = {"model.embed_tokens.comfy_quant": qt({"format": "int8_tensorwise"}),
                    "model.layers.0.mlp.down_proj.comfy_quant": qt({"format": "int8_tensorwise", "convrot": True,
                                                                    "convrot_groupsize": 256})}
    assert convrot_skip_reason(_save(tmp_path / "d.safetensors", text_encoder,
                                     {"minimax_h3_te": json.dumps({"num_hidden_layers": 50})})) is None


def test_dense_non_convrot_and_malformed_files_are_skipped(tmp_path):
    dense = _save(tmp_path / "dense.safetensors", {"blocks.0.ffn.0.weight": torch.zeros((1, 1))})
    int8 = _save(tmp_path / "int8.safetensors", {"blocks.0.ffn.0.comfy_quant": qt({"format": "int8_tensorwise"})})
    assert "does not contain supported ConvRot" in convrot_skip_reason(dense)
    assert "does not contain supported ConvRot" in convrot_skip_reason(int8)
    assert "unsupported file extension" in convrot_skip_reason(tmp_path / "model.ckpt")
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"\x01\x02")
    assert "could not read ConvRot metadata" in convrot_skip_reason(short)
    # A descriptor whose offsets point past the end of the file.
    body = json.dumps({"x.comfy_quant": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}).encode()
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(len(body).to_bytes(8, "little") + body)
    assert "outside the safetensors file" in convrot_skip_reason(bad)
