"""Minimal stand-in for comfy_kitchen (absent from this environment), built
from the names the reference's call sites use (backend.py:24-26, 98-145,
169-182; __init__.py:39-49): backends.eager.{int8_linear, quantization},
quantization.{int8_linear, _int8_matmul_accumulate, _apply_input_act,
_apply_residual, quantize_int8_rowwise}, registry.get_implementation.
Test infrastructure only."""
import sys
import types


def install(quantize=None):
    root = types.ModuleType("comfy_kitchen")
    backends = types.ModuleType("comfy_kitchen.backends")
    eager = types.ModuleType("comfy_kitchen.backends.eager")
    quant = types.ModuleType("comfy_kitchen.backends.eager.quantization")
    registry_mod = types.ModuleType("comfy_kitchen.registry")
    calls = {"original": 0, "input_act": 0, "residual": 0}

    def original_int8_linear(*args, **kwargs):
        calls["original"] += 1
        return "original"

    def apply_input_act(x, act, weight, eps):
        if act is None:
            return x
        calls["input_act"] += 1
        return x * 2                       # recognisable stand-in transformation

    def apply_residual(y, residual, scale):
        if residual is None:
            return y
        calls["residual"] += 1
        return y + residual

    quant.int8_linear = original_int8_linear
    quant._int8_matmul_accumulate = None
    quant._apply_input_act = apply_input_act
    quant._apply_residual = apply_residual
    quant.quantize_int8_rowwise = quantize
    eager.int8_linear = original_int8_linear
    eager.quantization = quant

    class Registry:
        def get_implementation(self, name, backend):
            return eager.int8_linear

    registry_mod.registry = Registry()
    root.backends = backends
    backends.eager = eager
    root.registry = registry_mod
    mods = {"comfy_kitchen": root, "comfy_kitchen.backends": backends,
            "comfy_kitchen.backends.eager": eager,
            "comfy_kitchen.backends.eager.quantization": quant,
            "comfy_kitchen.registry": registry_mod}
    saved = {k: sys.modules.get(k) for k in mods}
    sys.modules.update(mods)

    def uninstall():
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return types.SimpleNamespace(eager=eager, quant=quant, registry=registry_mod.registry,
                                 calls=calls, uninstall=uninstall)
