"""comfy-kitchen backend registration of the B200 ConvRot linears.

ComfyUI reaches the plugin's ConvRot linears through comfy-kitchen's backend registry:
the plugin registers its dispatcher module under ``BACKEND_NAME`` for the capabilities
``int8_linear``, ``convrot_w4a4_linear`` and (when kitchen's CUDA backend offers it)
``w4a8_int8_linear``, with per-argument constraints and call rules, and puts itself first
in the registry's priority list (comfyui_turing_utils/quantization/dispatch.py:939-1080).
This module does the same for the B200 dispatcher (``comfyui_turing_utils_b200.dispatch``):
same backend name, capability names, argument names and dtypes, rule outcomes and
priority order, with the device rule asking for a B200 instead of an sm75+ GPU.

comfy-kitchen is a third-party package the B200 build does not ship; ``register_backend``
imports it when installed, or takes a module with the same interface (``list_backends``,
``constraints``, ``registry``) as its argument.
"""

from __future__ import annotations

import logging
import sys
from types import ModuleType

import torch

from . import dispatch

LOG = logging.getLogger("comfyui-turing-utils")
BACKEND_NAME = dispatch.BACKEND_NAME

# Kitchen CUDA-backend capabilities the registration requires, and the optional one.
REQUIRED_CAPABILITIES = frozenset({"convrot_w4a4_linear", "int8_linear"})
CODEBOOK_CAPABILITY = "w4a8_int8_linear"


def _import_kitchen():
    try:
        import comfy_kitchen
        from comfy_kitchen import constraints as kitchen_constraints  # noqa: F401
        from comfy_kitchen.registry import registry  # noqa: F401
    except ImportError:
        return None
    return comfy_kitchen


def backend_available(kitchen: ModuleType) -> bool:
    """True when the registry lists BACKEND_NAME as available."""
    status = kitchen.list_backends().get(BACKEND_NAME, {})
    return bool(status.get("available", False))


def _call_rules(kitchen: ModuleType):
    """The reference's call rules (dispatch.py:976-1007), as closures over kitchen's
    ValidationResult."""
    result = kitchen.constraints.ValidationResult
    from comfyui_turing_utils_kernel import _C

    has_w4a8_kernel = hasattr(_C, "turing_w4a8_linear")
    has_codebook_w4a8_kernel = hasattr(_C, "turing_codebook_w4a8_linear")

    def require_convrot_256(kwargs):
        if kwargs.get("convrot") is not True:
            return result.fail("convrot", "staged INT8 requires ConvRot")
        if kwargs.get("convrot_groupsize") != dispatch.CONVROT_GROUP:
            return result.fail("convrot_groupsize", "staged INT8 requires group size 256")
        return result.ok()

    def require_w4_convrot_256(kwargs):
        if kwargs.get("convrot_groupsize") != dispatch.CONVROT_GROUP:
            return result.fail("convrot_groupsize", "W4 requires ConvRot group size 256")
        if kwargs.get("quant_group_size") != 64:
            return result.fail("quant_group_size", "W4 requires quantization group size 64")
        if kwargs.get("linear_dtype") not in {"int4", "int8"}:
            return result.fail("linear_dtype", "W4 requires int4 or int8 activation")
        if kwargs.get("linear_dtype") == "int8" and not has_w4a8_kernel:
            return result.fail("linear_dtype", "W4A8 kernel is unavailable")
        return result.ok()

    def require_codebook_w4a8(kwargs):
        if not has_codebook_w4a8_kernel:
            return result.fail("qdata", "codebook W4A8 kernel is unavailable")
        if kwargs.get("convrot_groupsize") != dispatch.CONVROT_GROUP:
            return result.fail("convrot_groupsize", "codebook W4A8 requires ConvRot group size 256")
        if kwargs.get("correction") is not None:
            return result.fail("correction", "codebook W4A8 fast path supports symmetric files only")
        if kwargs.get("codebook") is None:
            return result.fail("codebook", "codebook W4A8 requires a 16-entry codebook")
        return result.ok()

    return require_convrot_256, require_w4_convrot_256, require_codebook_w4a8


def build_operations(kitchen: ModuleType, with_codebook: bool) -> dict:
    """FunctionConstraints per capability (dispatch.py:1009-1073): argument dtypes, shape
    rules, CUDA as the default device, and the call rules above."""
    c = kitchen.constraints

    class SupportedB200Tensor(c.ShapeRule):
        def check(self, tensor: torch.Tensor) -> bool:
            return dispatch.is_supported_b200_device(tensor.device)

        def describe(self) -> str:
            return "tensor on an NVIDIA B200 (sm_100a) device"

    cuda_devices = frozenset({"cuda"})
    standard_floats = frozenset({torch.float32, torch.float16, torch.bfloat16})
    require_convrot_256, require_w4_convrot_256, require_codebook_w4a8 = _call_rules(kitchen)
    x_bf16 = c.ParamConstraint(dtypes=frozenset({torch.bfloat16}), shape_rules=(c.MinDims(2), SupportedB200Tensor()))
    operations = {
        "int8_linear": c.FunctionConstraints(
            params={
                "x": x_bf16,
                "weight": c.ParamConstraint(dtypes=frozenset({torch.int8}), shape_rules=(c.ExactDims(2),)),
                "weight_scale": c.ParamConstraint(dtypes=frozenset({torch.float32})),
                "bias": c.ParamConstraint(dtypes=standard_floats),
                "out_dtype": c.ParamConstraint(dtypes=standard_floats),
                "convrot": c.ParamConstraint(dtypes=frozenset({bool})),
                "convrot_groupsize": c.ParamConstraint(dtypes=frozenset({int})),
                "input_act": c.ParamConstraint(dtypes=frozenset({str, type(None)})),
            },
            default_devices=cuda_devices,
            call_rules=(require_convrot_256,),
        ),
        "convrot_w4a4_linear": c.FunctionConstraints(
            params={
                "x": x_bf16,
                "qweight": c.ParamConstraint(dtypes=frozenset({torch.int8}), shape_rules=(c.ExactDims(2),)),
                "wscales": c.ParamConstraint(dtypes=standard_floats, shape_rules=(c.ExactDims(1),)),
                "bias": c.ParamConstraint(dtypes=standard_floats),
                "convrot_groupsize": c.ParamConstraint(dtypes=frozenset({int})),
                "quant_group_size": c.ParamConstraint(dtypes=frozenset({int})),
                "linear_dtype": c.ParamConstraint(dtypes=frozenset({str})),
                "input_act": c.ParamConstraint(dtypes=frozenset({str, type(None)})),
            },
            default_devices=cuda_devices,
            call_rules=(require_w4_convrot_256,),
        ),
    }
    if with_codebook:
        operations[CODEBOOK_CAPABILITY] = c.FunctionConstraints(
            params={
                "x": x_bf16,
                "qdata": c.ParamConstraint(dtypes=frozenset({torch.int8}), shape_rules=(c.ExactDims(2),)),
                "s_rel": c.ParamConstraint(dtypes=frozenset({torch.float8_e4m3fn}), shape_rules=(c.ExactDims(2),)),
                "s_channel": c.ParamConstraint(dtypes=frozenset({torch.float32}), shape_rules=(c.ExactDims(1),)),
                "codebook": c.ParamConstraint(dtypes=frozenset({torch.float32})),
                "correction": c.ParamConstraint(dtypes=standard_floats),
                "bias": c.ParamConstraint(dtypes=standard_floats),
                "group_size": c.ParamConstraint(dtypes=frozenset({int})),
                "convrot_groupsize": c.ParamConstraint(dtypes=frozenset({int})),
                "out_dtype": c.ParamConstraint(dtypes=standard_floats),
            },
            default_devices=cuda_devices,
            call_rules=(require_codebook_w4a8,),
        )
    return operations


def register_backend(kitchen: ModuleType | None = None) -> bool:
    """Register the B200 dispatcher with comfy-kitchen's registry and make it the first
    backend tried.  Returns False when kitchen is not installed or its CUDA backend lacks
    the required capabilities; True when registered (or already available)."""
    if kitchen is None:
        kitchen = _import_kitchen()
        if kitchen is None:
            return False
    backends = kitchen.list_backends()
    cuda_capabilities = set(backends.get("cuda", {}).get("capabilities", ()))
    if not REQUIRED_CAPABILITIES.issubset(cuda_capabilities):
        return False
    if BACKEND_NAME in backends:
        return backend_available(kitchen)
    operations = build_operations(kitchen, CODEBOOK_CAPABILITY in cuda_capabilities)
    registry = kitchen.registry.registry
    registry.register(BACKEND_NAME, sys.modules[dispatch.__name__], operations)
    existing = list(getattr(registry, "_priority", ("cuda", "triton", "eager")))
    registry.set_priority([BACKEND_NAME, *(name for name in existing if name != BACKEND_NAME)])
    LOG.info("Registered the B200 ConvRot backend")
    return True
