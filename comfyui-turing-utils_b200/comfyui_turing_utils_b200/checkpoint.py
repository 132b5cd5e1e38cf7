"""ConvRot checkpoint metadata: which layers of a ComfyUI checkpoint run on which kernel.

Mirrors the load-time half of the reference plugin's ConvRot path
(comfyui_turing_utils/quantization/convrot.py:14-305): per-layer quantization configs
come from the safetensors header (``__metadata__["_quantization_metadata"]``, a
``{"layers": {name: config}}`` JSON) and from ``<layer>.comfy_quant`` uint8 tensors
holding JSON.  Each config is classified as W8 (``int8_tensorwise`` with ``convrot``),
W4 (``convrot_w4a4`` with ``linear_dtype`` int4 or int8) or grouped-codebook W4A8
(``asym_w4a8_int8``), legacy W8 spellings are normalised, and an optional
``force_int8_gemm`` rewrites every W4 layer to int8 activations.  The same rules and
error messages as the reference decide what a checkpoint may contain; ``kernel_for``
names the B200 op that serves each classified layer.
"""

from __future__ import annotations

import dataclasses
import json
import math
import struct
from pathlib import Path

import torch

MODEL_EXTENSIONS = {".safetensors", ".sft"}
W4_FORMAT = "convrot_w4a4"
CODEBOOK_W4_FORMAT = "asym_w4a8_int8"
W8_FORMAT = "int8_tensorwise"
LEGACY_W8_FORMAT = "int8_rowwise"
MAX_SAFETENSORS_HEADER_SIZE = 128 * 1024 * 1024
MAX_QUANT_CONFIG_SIZE = 1024 * 1024
QUANT_SUFFIX = ".comfy_quant"


@dataclasses.dataclass(frozen=True)
class ConvRotSummary:
    """Layer counts per (weight, activation) kind (convrot.py:23-28)."""

    w4a4: int = 0
    w4a8: int = 0
    codebook_w4a8: int = 0
    w8a8: int = 0


def _field(config: dict, name: str, default, layer: str):
    """A config value, read from the top level first and then from ``params``."""
    params = config.get("params", {})
    if not isinstance(params, dict):
        raise ValueError(f"ConvRot layer {layer} has non-object params metadata")
    return config[name] if name in config else params.get(name, default)


def classify_layer(config: dict, layer: str, force_int8_gemm: bool) -> tuple[str, str] | None:
    """convrot.py:40-101: ``(weight kind, activation dtype)`` of one layer config, None for
    a layer that is not ConvRot-quantized; raises ValueError for a config the path cannot
    run.  Legacy W8 configs (no format or ``int8_rowwise``, with ``convrot`` and
    ``per_row``) are rewritten in place to ``int8_tensorwise``."""
    if not isinstance(config, dict):
        raise ValueError(f"Quantization metadata for layer {layer} must be an object")
    fmt = config.get("format")
    if (fmt is None or fmt == LEGACY_W8_FORMAT) and _field(config, "convrot", False, layer) is True and \
            _field(config, "per_row", False, layer) is True:
        config["format"] = fmt = W8_FORMAT

    if fmt == W4_FORMAT:
        act = _field(config, "linear_dtype", "int4", layer)
        if act not in {"int4", "int8"}:
            raise ValueError(f"ConvRot W4 layer {layer} declares unsupported linear_dtype={act!r}; "
                             "expected 'int4' or 'int8'")
        return "w4", "int8" if force_int8_gemm else act

    if fmt == CODEBOOK_W4_FORMAT:
        if _field(config, "convrot", True, layer) is not True:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} must declare convrot=true")
        group = _field(config, "group_size", 16, layer)
        if not isinstance(group, int) or isinstance(group, bool) or group < 4:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} has invalid group_size={group!r}")
        if _field(config, "convrot_groupsize", 256, layer) != 256:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} requires convrot_groupsize=256")
        return "w4_codebook", "int8"

    convrot = _field(config, "convrot", False, layer)
    if not isinstance(convrot, bool):
        raise ValueError(f"Quantized layer {layer} has non-boolean convrot={convrot!r}")
    if not convrot:
        return None
    if fmt != W8_FORMAT:
        raise ValueError(f"ConvRot layer {layer} uses unsupported weight format {fmt!r}")
    act = _field(config, "linear_dtype", "int8", layer)
    if act not in {"int4", "int8"}:
        raise ValueError(f"ConvRot W8 layer {layer} declares unsupported linear_dtype={act!r}; expected 'int8'")
    if act != "int8" and not force_int8_gemm:
        raise ValueError(f"ConvRot W8 layer {layer} cannot use linear_dtype={act!r}; "
                         "W8 ConvRot supports INT8 activations only")
    return "w8", "int8"


def kernel_for(kind: tuple[str, str]) -> str:
    """The B200 op that serves a classified layer (the dispatch function names)."""
    return {
        ("w8", "int8"): "int8_linear",
        ("w4", "int8"): "convrot_w4a4_linear(linear_dtype='int8')",
        ("w4", "int4"): "convrot_w4a4_linear(linear_dtype='int4')",
        ("w4_codebook", "int8"): "codebook_w4a8_linear",
    }[kind]


def decode_quant_tensor(value: torch.Tensor, key: str) -> dict:
    """convrot.py:105-116: the JSON object a ``.comfy_quant`` uint8 tensor holds."""
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{key} must be a JSON byte tensor")
    try:
        config = json.loads(value.detach().cpu().numpy().tobytes())
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"{key} contains invalid quantization JSON") from exc
    if not isinstance(config, dict):
        raise ValueError(f"{key} quantization JSON must be an object")
    return config


def encode_quant_tensor(config: dict) -> torch.Tensor:
    """The inverse of decode_quant_tensor (convrot.py:119-120)."""
    return torch.tensor(list(json.dumps(config).encode("utf-8")), dtype=torch.uint8)


def configure_convrot_activation(state_dict: dict, metadata: dict | None, force_int8_gemm: bool,
                                 model_prefix: str | None = None) -> tuple[dict, ConvRotSummary]:
    """convrot.py:218-305: classify every ConvRot layer of a checkpoint (header configs
    and ``.comfy_quant`` tensors, optionally only names under ``model_prefix``), reject
    conflicting duplicates, apply ``force_int8_gemm`` (W4 layers to int8 activations,
    rewriting both metadata sources) and count the kinds.  Returns the updated metadata
    and the summary; ``state_dict``'s ``.comfy_quant`` tensors are rewritten in place."""
    if not isinstance(force_int8_gemm, bool):
        raise ValueError(f"force_int8_gemm must be boolean, got {force_int8_gemm!r}")
    metadata = dict(metadata or {})
    records: list[tuple[str, dict]] = []

    header = None
    raw = metadata.get("_quantization_metadata")
    if raw is not None:
        try:
            header = json.loads(raw)
        except (TypeError, json.JSONDecodeError) as exc:
            raise ValueError("Safetensors _quantization_metadata contains invalid JSON") from exc
        if not isinstance(header, dict) or not isinstance(header.get("layers"), dict):
            raise ValueError("Safetensors _quantization_metadata must contain a layers object")
        records += [(name, cfg) for name, cfg in header["layers"].items()
                    if model_prefix is None or name.startswith(model_prefix)]

    tensor_configs: dict[str, dict] = {}
    for key, value in state_dict.items():
        if not key.endswith(QUANT_SUFFIX):
            continue
        layer = key[: -len(QUANT_SUFFIX)]
        if model_prefix is not None and not layer.startswith(model_prefix):
            continue
        tensor_configs[key] = decode_quant_tensor(value, key)
        records.append((layer, tensor_configs[key]))

    kinds: dict[str, tuple[str, str]] = {}
    classified: list[tuple[dict, str]] = []
    for layer, config in records:
        kind = classify_layer(config, layer, force_int8_gemm)
        if kind is None:
            continue
        seen = kinds.setdefault(layer, kind)
        if seen != kind:
            raise ValueError(f"Conflicting ConvRot metadata for layer {layer}: "
                             f"{seen[0]}/{seen[1]} versus {kind[0]}/{kind[1]}")
        classified.append((config, kind[0]))
    if not classified:
        raise ValueError("The selected model does not contain supported ConvRot quantization metadata")

    if force_int8_gemm:
        for config, weight_kind in classified:
            if weight_kind != "w4_codebook":
                config["linear_dtype"] = "int8"
    if header is not None:
        metadata["_quantization_metadata"] = json.dumps(header)
    for key, config in tensor_configs.items():
        state_dict[key] = encode_quant_tensor(config)

    counts = {"w4a4": 0, "w4a8": 0, "codebook_w4a8": 0, "w8a8": 0}
    names = {("w4", "int4"): "w4a4", ("w4", "int8"): "w4a8", ("w4_codebook", "int8"): "codebook_w4a8",
             ("w8", "int8"): "w8a8"}
    for kind in kinds.values():
        counts[names[kind]] += 1
    return metadata, ConvRotSummary(**counts)


def _read_header(path: Path) -> tuple[dict, int, int]:
    """convrot.py:123-145: the safetensors JSON header, where tensor data starts, file size."""
    size = path.stat().st_size
    with path.open("rb") as handle:
        raw = handle.read(8)
        if len(raw) != 8:
            raise ValueError("file is too short to contain a safetensors header")
        header_size = struct.unpack("<Q", raw)[0]
        if header_size == 0 or header_size > MAX_SAFETENSORS_HEADER_SIZE:
            raise ValueError(f"invalid safetensors header size {header_size}")
        data_start = 8 + header_size
        if data_start > size:
            raise ValueError(f"safetensors header ends at byte {data_start}, beyond file size {size}")
        raw_header = handle.read(header_size)
    try:
        header = json.loads(raw_header)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError("safetensors header contains invalid JSON") from exc
    if not isinstance(header, dict):
        raise ValueError("safetensors header must be an object")
    return header, data_start, size


def _read_tensor_config(handle, info: dict, key: str, data_start: int, size: int) -> dict:
    """convrot.py:148-191: one ``.comfy_quant`` tensor's JSON, read from the file with
    every descriptor field checked before any byte is read."""
    if not isinstance(info, dict):
        raise ValueError(f"{key} has an invalid safetensors tensor descriptor")
    if info.get("dtype") != "U8":
        raise ValueError(f"{key} must use U8 storage")
    shape, offsets = info.get("shape"), info.get("data_offsets")
    if (not isinstance(shape, list)
            or any(not isinstance(d, int) or isinstance(d, bool) or d < 0 for d in shape)
            or not isinstance(offsets, list) or len(offsets) != 2
            or any(not isinstance(o, int) or isinstance(o, bool) for o in offsets)):
        raise ValueError(f"{key} has invalid shape or data offsets")
    begin, end = offsets
    length = end - begin
    if length != math.prod(shape):
        raise ValueError(f"{key} byte length does not match its U8 shape")
    if length > MAX_QUANT_CONFIG_SIZE:
        raise ValueError(f"{key} is too large to be quantization JSON")
    if begin < 0 or data_start + end < data_start + begin or data_start + end > size:
        raise ValueError(f"{key} data offsets are outside the safetensors file")
    handle.seek(data_start + begin)
    raw = handle.read(length)
    if len(raw) != length:
        raise ValueError(f"{key} tensor data is truncated")
    try:
        config = json.loads(raw)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"{key} contains invalid quantization JSON") from exc
    if not isinstance(config, dict):
        raise ValueError(f"{key} quantization JSON must be an object")
    return config


def convrot_skip_reason(path: str | Path) -> str | None:
    """convrot.py:194-215: None when the file holds at least one ConvRot layer (header or
    tensor metadata, classified as with ``force_int8_gemm``), else the reason to skip it.
    Reads only the header and the small ``.comfy_quant`` tensors."""
    path = Path(path)
    if path.suffix.lower() not in MODEL_EXTENSIONS:
        return f"unsupported file extension {path.suffix!r}"
    try:
        index, data_start, size = _read_header(path)
        meta = index.get("__metadata__", {})
        if not isinstance(meta, dict):
            return "safetensors __metadata__ must be an object"
        raw = meta.get("_quantization_metadata")
        if raw is not None:
            quantization = json.loads(raw)
            if not isinstance(quantization, dict) or not isinstance(quantization.get("layers"), dict):
                return "safetensors _quantization_metadata must contain a layers object"
            if any(classify_layer(cfg, name, True) is not None for name, cfg in quantization["layers"].items()):
                return None
        with path.open("rb") as handle:
            for key, info in index.items():
                if key == "__metadata__" or not key.endswith(QUANT_SUFFIX):
                    continue
                config = _read_tensor_config(handle, info, key, data_start, size)
                if classify_layer(config, key[: -len(QUANT_SUFFIX)], True) is not None:
                    return None
    except Exception as exc:  # any malformed file is a reason to skip it, like the reference
        return f"could not read ConvRot metadata ({exc})"
    return "does not contain supported ConvRot quantization metadata"
