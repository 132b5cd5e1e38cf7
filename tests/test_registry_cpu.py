"""comfy-kitchen registration of the B200 ConvRot backend, against a minimal stand-in for
the kitchen registry (comfy-kitchen itself is a third-party package the build does not
ship).  The checks restate what the reference's register_backend does
(comfyui_turing_utils/quantization/dispatch.py:939-1080): the capability gate, the
already-registered path, the per-operation constraints and call rules, the dispatcher
module registered, and the backend first in priority."""

from types import ModuleType, SimpleNamespace

import pytest
import torch


def fake_kitchen(capabilities=("int8_linear", "convrot_w4a4_linear"), registered=None):
    """A module with the kitchen interface register_backend uses."""
    class ValidationResult(SimpleNamespace):
        @classmethod
        def ok(cls):
            return cls(ok=True, param=None, reason=None)

        @classmethod
        def fail(cls, param, reason):
            return cls(ok=False, param=param, reason=reason)

    class ShapeRule:
        def check(self, tensor):
            raise NotImplementedError

    class MinDims(ShapeRule):
        def __init__(self, n):
            self.n = n

        def check(self, tensor):
            return tensor.dim() >= self.n

    class ExactDims(ShapeRule):
        def __init__(self, n):
            self.n = n

        def check(self, tensor):
            return tensor.dim() == self.n

    class ParamConstraint(SimpleNamespace):
        def __init__(self, dtypes=frozenset(), shape_rules=()):
            super().__init__(dtypes=dtypes, shape_rules=shape_rules)

    class FunctionConstraints(SimpleNamespace):
        def __init__(self, params, default_devices, call_rules=()):
            super().__init__(params=params, default_devices=default_devices, call_rules=call_rules)

    class Registry:
        def __init__(self):
            self.backends = {}
            self._priority = ("cuda", "triton", "eager")

        def register(self, name, module, operations):
            self.backends[name] = (module, operations)

        def set_priority(self, names):
            self._priority = tuple(names)

    registry = Registry()
    kitchen = ModuleType("comfy_kitchen")
    kitchen.constraints = SimpleNamespace(ValidationResult=ValidationResult, ShapeRule=ShapeRule, MinDims=MinDims,
                                          ExactDims=ExactDims, ParamConstraint=ParamConstraint,
                                          FunctionConstraints=FunctionConstraints)
    kitchen.registry = SimpleNamespace(registry=registry)

    def list_backends():
        out = {"cuda": {"available": True, "capabilities": list(capabilities)}}
        for name in registry.backends:
            out[name] = {"available": True}
        if registered is not None:
            out.update(registered)
        return out

    kitchen.list_backends = list_backends
    return kitchen


@pytest.fixture
def reg():
    from comfyui_turing_utils_b200 import registry

    return registry


def test_no_kitchen_means_no_registration(reg, monkeypatch):
    monkeypatch.setattr(reg, "_import_kitchen", lambda: None)
    assert reg.register_backend() is False


def test_missing_cuda_capabilities_refuse_registration(reg):
    kitchen = fake_kitchen(capabilities=("int8_linear",))
    assert reg.register_backend(kitchen) is False
    assert kitchen.registry.registry.backends == {}


def test_registration_puts_the_backend_first_with_the_dispatcher(reg):
    from comfyui_turing_utils_b200 import dispatch

    kitchen = fake_kitchen()
    assert reg.register_backend(kitchen) is True
    r = kitchen.registry.registry
    module, ops = r.backends["turing_utils_sm75"]
    assert module is dispatch
    assert set(ops) == {"int8_linear", "convrot_w4a4_linear"}
    assert r._priority == ("turing_utils_sm75", "cuda", "triton", "eager")
    # Every registered capability is a function of the dispatcher with those argument names.
    import inspect

    for name, constraints in ops.items():
        params = inspect.signature(getattr(dispatch, name)).parameters
        assert set(constraints.params) <= set(params), name
        assert constraints.default_devices == frozenset({"cuda"})


def test_codebook_capability_is_registered_only_when_kitchen_offers_it(reg):
    import inspect

    from comfyui_turing_utils_b200 import dispatch

    kitchen = fake_kitchen(capabilities=("int8_linear", "convrot_w4a4_linear", "w4a8_int8_linear"))
    assert reg.register_backend(kitchen)
    ops = kitchen.registry.registry.backends["turing_utils_sm75"][1]
    assert "w4a8_int8_linear" in ops
    assert ops["w4a8_int8_linear"].params["s_rel"].dtypes == frozenset({torch.float8_e4m3fn})
    # The dispatcher answers to every registered name (w4a8_int8_linear is the codebook op).
    assert dispatch.w4a8_int8_linear is dispatch.codebook_w4a8_linear
    for name, constraints in ops.items():
        assert set(constraints.params) <= set(inspect.signature(getattr(dispatch, name)).parameters), name


def test_already_registered_returns_availability(reg):
    kitchen = fake_kitchen(registered={"turing_utils_sm75": {"available": False}})
    assert reg.register_backend(kitchen) is False
    kitchen = fake_kitchen(registered={"turing_utils_sm75": {"available": True}})
    assert reg.register_backend(kitchen) is True
    assert kitchen.registry.registry.backends == {}  # nothing registered twice


def test_call_rules_restate_the_reference_conditions(reg):
    kitchen = fake_kitchen(capabilities=("int8_linear", "convrot_w4a4_linear", "w4a8_int8_linear"))
    ops = reg.build_operations(kitchen, with_codebook=True)
    (w8,) = ops["int8_linear"].call_rules
    assert w8({"convrot": True, "convrot_groupsize": 256}).ok
    assert w8({"convrot": False, "convrot_groupsize": 256}).param == "convrot"
    assert w8({"convrot": True, "convrot_groupsize": 128}).param == "convrot_groupsize"
    (w4,) = ops["convrot_w4a4_linear"].call_rules
    good = {"convrot_groupsize": 256, "quant_group_size": 64, "linear_dtype": "int4"}
    assert w4(good).ok and w4({**good, "linear_dtype": "int8"}).ok
    assert w4({**good, "quant_group_size": 32}).param == "quant_group_size"
    assert w4({**good, "linear_dtype": "fp8"}).param == "linear_dtype"
    (cb,) = ops["w4a8_int8_linear"].call_rules
    okc = {"convrot_groupsize": 256, "correction": None, "codebook": torch.zeros(16)}
    assert cb(okc).ok
    assert cb({**okc, "correction": torch.zeros(1)}).param == "correction"
    assert cb({**okc, "codebook": None}).param == "codebook"


def test_shape_rules_require_2d_bf16_on_a_b200(reg):
    kitchen = fake_kitchen()
    ops = reg.build_operations(kitchen, with_codebook=False)
    x = ops["int8_linear"].params["x"]
    assert x.dtypes == frozenset({torch.bfloat16})
    min_dims, device_rule = x.shape_rules
    assert min_dims.check(torch.zeros(2, 3)) and not min_dims.check(torch.zeros(3))
    assert not device_rule.check(torch.zeros(2, 3))  # a CPU tensor is never accepted
    assert "B200" in device_rule.describe()
