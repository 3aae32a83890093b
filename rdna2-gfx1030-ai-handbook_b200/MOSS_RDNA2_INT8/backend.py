"""Production MOSS INT8 eager export on B200 (drop-in for the reference's
production/MOSS_RDNA2_INT8/backend.py:1-204).

Same public functions and install protocol as rdna2_ops.comfy_int8, with
this module's own installation state and statistics (the reference also
keeps two independent copies).  The linear itself runs on the library's
rotation+quantize prologue and tcgen05 INT8 GEMM with the Kitchen epilogue
order (x_scale * w_scale, cast, then + bias in the output dtype).
"""
import torch

from rdna2_ops.comfy_int8 import KitchenInt8Binding

_binding = KitchenInt8Binding()


def int8_linear(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16, convrot=False,
                convrot_groupsize=256, input_act=None, input_act_weight=None, input_act_eps=0.0,
                residual=None, residual_scale=None):
    """Pinned eager INT8 linear semantics on the B200 kernels."""
    return _binding.int8_linear(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize,
                                input_act, input_act_weight, input_act_eps, residual, residual_scale)


def install_backend(strided_int8_matmul):
    """Replace only Kitchen's eager export int8_linear; verified through the
    registry; call between workloads."""
    _binding.install_backend(strided_int8_matmul, int8_linear)


def disable_backend():
    """Restore the original eager export; refuses to overwrite another patch."""
    _binding.disable_backend(int8_linear)


def get_stats():
    return _binding.get_stats()


def reset_stats():
    _binding.reset_stats()
