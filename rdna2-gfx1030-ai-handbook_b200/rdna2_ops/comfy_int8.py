"""Kitchen eager INT8 linear on the B200 kernels, without a weight copy.

Drop-in for the reference's rdna2_ops/comfy_int8.py and the production node's
MOSS_RDNA2_INT8/backend.py (both at lines 1-204): the same public functions
(int8_linear, install_backend, disable_backend, get_stats, reset_stats,
kitchen_int8_without_transpose_copy), the same install/verify/restore
protocol against comfy_kitchen's eager export and registry, the same
optional statistics (MOSS_RDNA2_INT8_STATS=1), and the same epilogue order:
float(acc) * (x_scale * w_scale) cast to out_dtype, then + bias in out_dtype
(backend.py:128-143).

Differences on B200: the whole linear -- ConvRot block-Hadamard, per-token
INT8 quantization, INT8 GEMM on tcgen05, scale/cast/bias -- runs in the
library's two kernels (b2_quant_linear); fp16/bf16 inputs and outputs are
accelerated too (the reference falls back to Kitchen for them,
backend.py:90-97).  Kitchen's input activation and residual helpers are
called as they are.  Weights are read through their stored [N,K] layout on
every call; nothing is cached.
"""
from __future__ import annotations

import os
from contextlib import contextmanager
from threading import Lock

import torch

from .qlinear import w8a8_linear


class KitchenInt8Binding:
    """One installable replacement of Kitchen's eager int8_linear export."""

    def __init__(self):
        self._matmul = None
        self._original_export = None
        self._installed = False
        self._installation_lock = Lock()
        self._stats_enabled = os.environ.get("MOSS_RDNA2_INT8_STATS", "0") == "1"
        self._stats_lock = Lock()
        self._calls = 0
        self._layouts = {}
        self._context_lock = Lock()

    # ------------------------------------------------------------ stats
    def _record_layout(self, weight):
        rhs = weight.T
        key = (tuple(weight.shape), tuple(weight.stride()), tuple(rhs.stride()), str(weight.device))
        with self._stats_lock:
            self._calls += 1
            self._layouts[key] = self._layouts.get(key, 0) + 1

    def get_stats(self):
        """Successful GEMM counts/layouts when MOSS_RDNA2_INT8_STATS=1; never
        retains tensors or logs per call."""
        with self._stats_lock:
            return {
                "enabled": self._stats_enabled,
                "calls": self._calls,
                "weight_layouts": [
                    {"shape": shape, "weight_stride": stride, "rhs_stride": rhs_stride,
                     "device": device, "dtype": "torch.int8", "calls": count}
                    for (shape, stride, rhs_stride, device), count in self._layouts.items()
                ],
            }

    def reset_stats(self):
        with self._stats_lock:
            self._calls = 0
            self._layouts.clear()

    # ----------------------------------------------------------- linear
    def int8_linear(self, x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16, convrot=False,
                    convrot_groupsize=256, input_act=None, input_act_weight=None, input_act_eps=0.0,
                    residual=None, residual_scale=None):
        if self._matmul is None:
            raise RuntimeError("Install the MOSS INT8 eager export before calling it")
        if input_act is not None:
            x = _kitchen().quantization._apply_input_act(x, input_act, input_act_weight, input_act_eps)
        if x.shape[-1] != weight.shape[-1]:
            raise ValueError(
                f"Input and weight inner dimensions must match, got {x.shape[-1]} and {weight.shape[-1]}")
        weight = weight.to(device=x.device)
        weight_scale = weight_scale.to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
        if weight_scale.numel() not in (1, weight.shape[0]):
            raise ValueError(
                f"INT8 weight scale must be scalar or per-output-channel, got {tuple(weight_scale.shape)} "
                f"for weight shape {tuple(weight.shape)}")
        if convrot and x.shape[-1] % convrot_groupsize != 0:
            raise ValueError(
                f"ConvRot group size {convrot_groupsize} does not divide input features {x.shape[-1]}")
        if bias is not None:
            bias = bias.to(device=x.device).reshape(-1)
            if not bias.is_contiguous():
                bias = bias.contiguous()
        result = w8a8_linear(x, weight, weight_scale, bias,
                             rotation_block=convrot_groupsize if convrot else None,
                             out_dtype=out_dtype, epilogue="kitchen")
        if self._stats_enabled:
            self._record_layout(weight)
        if residual is not None:
            result = _kitchen().quantization._apply_residual(result, residual, residual_scale)
        return result

    # ------------------------------------------------- install / remove
    def install_backend(self, strided_int8_matmul, linear):
        """Replace only Kitchen's eager module export `int8_linear` with `linear`
        (reference backend.py:148-188); registry identity, priorities and
        capabilities are untouched and the swap is verified through
        registry.get_implementation."""
        if not callable(strided_int8_matmul):
            raise TypeError("strided_int8_matmul must be callable")
        eager_backend, eager, registry = _kitchen_parts()
        with self._installation_lock:
            if self._installed:
                if self._matmul is not strided_int8_matmul:
                    raise RuntimeError("MOSS INT8 export is already bound to a different GEMM")
                if eager_backend.int8_linear is not linear:
                    raise RuntimeError("Kitchen eager int8_linear changed while this patch was installed")
                return
            if eager._int8_matmul_accumulate is not strided_int8_matmul:
                raise RuntimeError("Install the B200 INT8 GEMM as Kitchen's accumulator first")
            original = eager.int8_linear
            if eager_backend.int8_linear is not original:
                raise RuntimeError("Expected Kitchen's unmodified eager int8_linear export")
            if registry.get_implementation("int8_linear", backend="eager") is not original:
                raise RuntimeError("Kitchen eager dispatch does not resolve the expected export")
            self._original_export = original
            self._matmul = strided_int8_matmul
            try:
                eager_backend.int8_linear = linear
                if registry.get_implementation("int8_linear", backend="eager") is not linear:
                    raise RuntimeError("Kitchen eager dispatch did not pick up its replacement export")
            except Exception:
                eager_backend.int8_linear = original
                self._original_export = None
                self._matmul = None
                raise
            self._installed = True

    def disable_backend(self, linear):
        """Restore the original export (reference backend.py:191-204); refuses
        to overwrite another patch's export."""
        eager_backend, _, _ = _kitchen_parts()
        with self._installation_lock:
            if not self._installed:
                return
            if eager_backend.int8_linear is not linear:
                raise RuntimeError("Kitchen eager int8_linear changed; refusing to overwrite it")
            eager_backend.int8_linear = self._original_export
            self._installed = False

    @contextmanager
    def scoped(self, strided_int8_matmul, linear):
        """Scoped install (reference comfy_int8.py:211-227); nested or concurrent
        contexts are rejected."""
        if not self._context_lock.acquire(blocking=False):
            raise RuntimeError("Nested or concurrent Kitchen INT8 contexts are unsupported")
        try:
            self.install_backend(strided_int8_matmul, linear)
            try:
                yield
            finally:
                self.disable_backend(linear)
        finally:
            self._context_lock.release()


def _kitchen():
    try:
        import comfy_kitchen.backends.eager as eager_backend
    except ImportError as exc:  # pragma: no cover - depends on the host install
        raise RuntimeError("comfy_kitchen is required for input activations, residuals and "
                           "backend installation") from exc
    return eager_backend


def _kitchen_parts():
    eager_backend = _kitchen()
    from comfy_kitchen.backends.eager import quantization as eager
    from comfy_kitchen.registry import registry
    return eager_backend, eager, registry


def module_api(binding):
    """The reference module's public functions (comfy_int8.py:71-227,
    production/MOSS_RDNA2_INT8/backend.py:71-204) bound to one
    KitchenInt8Binding: (int8_linear, install_backend, disable_backend,
    get_stats, reset_stats, kitchen_int8_without_transpose_copy).  Each module
    that exposes the API owns its binding, so installation state and
    statistics stay separate per module as in the reference."""

    def int8_linear(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16, convrot=False,
                    convrot_groupsize=256, input_act=None, input_act_weight=None, input_act_eps=0.0,
                    residual=None, residual_scale=None):
        """Kitchen's eager INT8 linear semantics on the B200 kernels: input
        activation, ConvRot, per-token INT8, GEMM, (acc*(sx*sw)).to(out) + bias,
        residual."""
        return binding.int8_linear(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize,
                                   input_act, input_act_weight, input_act_eps, residual, residual_scale)

    def install_backend(strided_int8_matmul):
        """Replace only Kitchen's eager int8_linear export, verified through
        the registry; call between workloads."""
        binding.install_backend(strided_int8_matmul, int8_linear)

    def disable_backend():
        """Restore the original export; refuses to overwrite another patch."""
        binding.disable_backend(int8_linear)

    @contextmanager
    def kitchen_int8_without_transpose_copy(strided_int8_matmul):
        """Scoped install; nested or concurrent contexts are rejected."""
        with binding.scoped(strided_int8_matmul, int8_linear):
            yield

    return (int8_linear, install_backend, disable_backend, binding.get_stats, binding.reset_stats,
            kitchen_int8_without_transpose_copy)


_binding = KitchenInt8Binding()
(int8_linear, install_backend, disable_backend, get_stats, reset_stats,
 kitchen_int8_without_transpose_copy) = module_api(_binding)
