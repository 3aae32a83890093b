"""B200 (sm_100a) drop-in for the reference's quantized-linear operators.

Same module and function names as the reference package rdna2_ops
(unixyo/rdna2-gfx1030-ai-handbook, rdna2-ops/rdna2_ops/): int8_gemm,
comfy_int8, int4_weight_gemm_v07, fp8_weight_gemm_v06.  Kernels are
hand-written CUDA for sm_100a in librdna2_b200.so (C ABI:
include/b2_qlinear.h); this package is the host-side mirror that validates
arguments like the reference and launches on torch's current stream.
"""
from .qlinear import act_quant, fp8_linear, quantize_weight, w8a8_linear
from .int8_gemm import int8_gemm_dequant, int8_matmul

__all__ = ["act_quant", "quantize_weight", "w8a8_linear", "fp8_linear", "int8_matmul",
           "int8_gemm_dequant"]
__version__ = "0.1.0"
