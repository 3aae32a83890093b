"""FP8 weight GEMM on sm_100a (drop-in for the reference's
rdna2_ops/fp8_weight_gemm_v06.py).

Reference contract (fp8_weight_gemm_v06.py:1-12, 140-206): fp16 activation
A[M,K] times an *unscaled* e4m3fn/e5m2 weight W[N,K], fp16 output, methods
upcast / decode / prepared_fp16 / fused_dot2 / int8 / prepared_int8;
prepared weights are explicit caller-owned tensors; eager inference only.

On B200 every method runs on this library's kernels:
  upcast, decode, fused_dot2  exact fp8 -> fp16 decode kernel, then the
                              tcgen05 kind::f16 GEMM (fp32 accumulation)
  prepared_fp16               the kind::f16 GEMM on the caller's fp16 weight
  int8, prepared_int8         the reference row quantizer (_quant_rows
                              semantics, mode 2 of b2_act_quant) on A and W,
                              then the tcgen05 kind::i8 GEMM with the
                              separate fp32 epilogue, cast to fp16
  scaled_e4m3 (new)           the north-star FP8 path: A -> e4m3 with a
                              per-token scale, W pre-scaled e4m3 with a
                              per-channel fp32 scale, tcgen05 kind::f8f6f4,
                              y = acc * (sa * sw) (+bias) cast to A's dtype
"""
from __future__ import annotations

import torch

from . import _native as nat
from .int4_weight_gemm_v07 import dense_linear
from .int8_gemm import int8_gemm_dequant
from .qlinear import fp8_linear, quantize_weight

_FP8 = (torch.float8_e4m3fn, torch.float8_e5m2)
METHODS = ("upcast", "decode", "prepared_fp16", "fused_dot2", "int8", "prepared_int8", "scaled_e4m3")


def _weight(w):
    if w.ndim != 2 or w.dtype not in _FP8:
        raise TypeError("Weight must be a plain unscaled FP8 [N,K] tensor")
    nat.require_device(w)
    if min(w.shape) <= 0 or min(w.stride()) <= 0 or sum((n - 1) * s for n, s in zip(w.shape, w.stride())) >= 2**31:
        raise ValueError("Nonempty positive strides and signed-32-bit address span required")


def decode_fp8_weight(w, *, out_dtype=torch.float16, metadata=None):
    """Decode every storage value; all finite FP8 values are exact in fp16
    (reference fp8_weight_gemm_v06.py:109-124)."""
    _weight(w)
    if out_dtype not in (torch.float16, torch.float32):
        raise TypeError("Decode output must be FP16 or FP32")
    n, k = w.shape
    if w.stride(1) != 1:
        w = w.contiguous()
    out = torch.empty((n, k), dtype=out_dtype, device=w.device)
    nat.check(nat.library().b2_fp8_decode(
        w.data_ptr(), nat.DTYPE_CODE[w.dtype], n, k, w.stride(0) if n > 1 else k,
        nat.DTYPE_CODE[out_dtype], out.data_ptr(), k, nat.stream_ptr(w.device)), "b2_fp8_decode")
    if metadata is not None:
        metadata.update(method="software_decode", output_dtype=str(out_dtype),
                        kernel="fp8_decode_kernel")
    return out


def _quant_rows(x):
    """Reference _quant_rows semantics on the device (b2_act_quant quant=2)."""
    m, k = x.shape
    if x.stride(1) != 1:
        x = x.contiguous()
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    nat.check(nat.library().b2_act_quant(
        x.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k, x.stride(0) if m > 1 else k, 0, 2, q.data_ptr(),
        k, s.data_ptr(), nat.stream_ptr(x.device)), "b2_act_quant")
    return q, s


def prepare_int8_weight(w):
    """Caller-owned (INT8 [N,K], FP32 per-output scale), no hidden cache."""
    _weight(w)
    if w.shape[1] > 32768:
        raise ValueError("This bounded row quantizer supports K<=32768")
    return _quant_rows(w)


def prepare_scaled_e4m3_weight(w):
    """Per-output-channel e4m3 weight for method="scaled_e4m3": scale =
    absmax/448 of each row (fp32), codes RNE with saturation."""
    if w.ndim != 2 or not w.is_floating_point():
        raise TypeError("Floating [N,K] weight required")
    return quantize_weight(w, quant="e4m3")


def fp8_weight_gemm(a, w, *, bias=None, method="upcast", prepared=None, tile=(64, 64, 32),
                    num_warps=4, metadata=None, w_scale=None):
    """fp16 A[M,K] x FP8 weight[N,K] -> fp16 [M,N] (reference
    fp8_weight_gemm_v06.py:140-206).  method="scaled_e4m3" also accepts bf16
    A and requires `w_scale` (per-channel fp32) for an e4m3 weight."""
    if method not in METHODS:
        raise ValueError("Unknown method: " + str(method))
    _weight(w)
    half_ok = (torch.float16, torch.bfloat16) if method == "scaled_e4m3" else (torch.float16,)
    if a.ndim != 2 or a.shape[1] != w.shape[1] or a.dtype not in half_ok or a.device != w.device:
        raise ValueError("FP16 [M,K] activation and matching FP8 [N,K] weight required")
    nat.eager_only(a, w)
    if torch.is_autocast_enabled("cuda"):
        raise ValueError("Only explicit eager inference is supported")
    if min(a.shape) <= 0 or min(a.stride()) <= 0 or sum((n - 1) * s for n, s in zip(a.shape, a.stride())) >= 2**31:
        raise ValueError("Nonempty positive-stride activation required")
    m, k = a.shape
    n = w.shape[0]
    if m * n >= 2**31:
        raise ValueError("Output exceeds supported indexing span")
    if bias is not None and (bias.shape != (n,) or bias.device != a.device or bias.dtype != a.dtype
                             or not bias.is_contiguous()):
        raise ValueError("Bias must be a contiguous vector of length N in the activation dtype")
    if method in ("upcast", "decode", "fused_dot2"):
        out = dense_linear(a.contiguous(), decode_fp8_weight(w), bias)
        if metadata is not None:
            metadata.update(method=method, kernel="fp8_decode_kernel + qgemm<kind::f16>")
        return out
    if method == "prepared_fp16":
        if prepared is None or prepared.shape != w.shape or prepared.device != w.device or prepared.dtype != a.dtype:
            raise ValueError("Provide the current FP16 prepared weight")
        return dense_linear(a.contiguous(), prepared.contiguous(), bias)
    if method in ("int8", "prepared_int8"):
        if method == "prepared_int8" and (not isinstance(prepared, tuple) or len(prepared) != 2):
            raise ValueError("Provide the current (INT8 weight, FP32 row scale)")
        qw, sw = prepare_int8_weight(w) if method == "int8" else prepared
        if (qw.shape != w.shape or qw.device != w.device or qw.dtype != torch.int8
                or sw.shape != (n,) or sw.device != w.device or sw.dtype != torch.float32):
            raise ValueError("Invalid prepared INT8 weight/scales")
        if k > 32768:
            raise ValueError("This bounded row quantizer supports K<=32768")
        qa, sa = _quant_rows(a)
        result = int8_gemm_dequant(qa, qw.T, sa, sw, bias, tile=(64, 128, 64), num_warps=4,
                                   num_stages=2, group_m=8)
        if metadata is not None:
            metadata.update(method=method, kernel="act_quant(mode 2) + qgemm<kind::i8>")
        return result.to(a.dtype)
    # scaled_e4m3
    if w.dtype != torch.float8_e4m3fn or w_scale is None:
        raise ValueError("scaled_e4m3 needs an e4m3fn weight and its per-channel fp32 w_scale")
    return fp8_linear(a, w, w_scale, bias, out_dtype=a.dtype)
