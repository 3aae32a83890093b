"""INT8 GEMM with an optional fused FP32 dequantization epilogue, on sm_100a.

Public surface of the reference module rdna2_ops/int8_gemm.py (names,
signatures and exception classes): int8_matmul (:195-200), int8_gemm_dequant
(:203-214), moss_int8_gemm_candidate (:217-271), qwen_int8_gemm_candidate
(:274-330).  The contraction runs on tcgen05 kind::i8 tensor cores with
TMEM accumulators (csrc/qgemm.cu, C ABI b2_qgemm) instead of the gfx1030 dot4
Triton kernels _int8_dot_dequant / _int8_dot_dequant_wrapped (:19-123).

Numerical contract kept from the reference:
  * epilogue value float(acc) * (row_scale * col_scale) (+ bias) in fp32
    (:53-63); rounding="separate" rounds the product and the sum separately,
    rounding="fused" uses one FMA (:191);
  * B is read through its strides, so the weight.T view needs no copy
    (:39-40); layouts the TMA cannot address are repacked per call;
  * a fresh output per call (:178).
The Triton launch keywords (tile, num_warps, num_stages, group_m, wrapped,
partial_dot) are checked for the reference's domains and otherwise unused.
Extension: `out_dtype` (fp32 default) casts in the epilogue to fp16/bf16.
"""
from __future__ import annotations

import sys
from contextlib import contextmanager

import torch

from . import _args
from . import _native as nat
from ._args import require
from ._patch import CandidateStats, scoped_patch
from .qlinear import qgemm_raw, w8a8_linear

_ROUNDING = {"separate": nat.EPI_SEPARATE, "fused": nat.EPI_FMA}
_KERNEL_INFO = {"name": "qgemm (tcgen05 kind::i8)", "arch": "sm_100a"}


def _run(a, b, scales, bias, *, rounding, out_dtype, tuning, wrapped, partial_dot, return_kernel):
    """Shared body of the two GEMM entry points.  `scales` is None for the
    raw INT32 product, else the (row, column) fp32 scale pair."""
    m, n, _, dev = _args.int8_operands(a, b)
    _args.tuning_keywords(*tuning)
    _args.eager_call()
    require(wrapped or not partial_dot, ValueError,
            "partial_dot requires the explicitly wrapped-load variant")
    require(rounding in _ROUNDING, ValueError, f"rounding must be 'separate' or 'fused', got {rounding!r}")
    if scales is None:
        out = torch.empty((m, n), device=dev, dtype=torch.int32)
        epilogue, a_scale, b_scale, bias = nat.EPI_NONE, None, None, None
    else:
        a_scale, b_scale = scales
        _args.fp32_vector(a_scale, m, "a_scale", dev)
        _args.fp32_vector(b_scale, n, "b_scale", dev, scalar_ok=True)
        _args.bias_vector(bias, n, dev)
        _args.no_autograd(a_scale, b_scale, bias)
        _args.output_dtype(out_dtype)
        out = torch.empty((m, n), device=dev, dtype=out_dtype)
        epilogue = _ROUNDING[rounding]
    if m and n:
        qgemm_raw(nat.KIND_I8, a, b.T, a_scale, b_scale, bias, epilogue, out)
    if return_kernel:
        return out, (dict(_KERNEL_INFO) if m and n else None)
    return out


def int8_matmul(a, b, *, tile=(32, 64, 64), num_warps=4, num_stages=1,
                group_m=4, return_kernel=False, wrapped=False, partial_dot=False):
    """Exact INT8 x INT8 -> INT32 product of a [M,K] and b [K,N] (any
    non-negative strides; the weight.T view of an [N,K] weight is read in
    place)."""
    return _run(a, b, None, None, rounding="separate", out_dtype=torch.int32,
                tuning=(tile, num_warps, num_stages, group_m), wrapped=wrapped,
                partial_dot=partial_dot, return_kernel=return_kernel)


def int8_gemm_dequant(a, b, a_scale, b_scale, bias=None, *, tile=(32, 64, 64),
                      num_warps=4, num_stages=1, group_m=4,
                      rounding="separate", return_kernel=False, wrapped=False, partial_dot=False,
                      out_dtype=torch.float32):
    """INT8 GEMM with the row x column (or row x scalar) fp32 dequantization
    and optional bias applied in the GEMM's epilogue.  Operands are already
    quantized; finite scales and bias are the caller's precondition."""
    return _run(a, b, (a_scale, b_scale), bias, rounding=rounding, out_dtype=out_dtype,
                tuning=(tile, num_warps, num_stages, group_m), wrapped=wrapped,
                partial_dot=partial_dot, return_kernel=return_kernel)


# ------------------------------------------------------------------ MOSS
def _moss_fused_linear(x, weight, weight_scale, bias, out_dtype, rotation_block):
    """Kitchen's int8_linear contract (ConvRot, per-token quantization, GEMM,
    fp32 "separate" epilogue with an fp32 bias) as one b2_quant_linear call."""
    k = x.shape[-1]
    require(k == weight.shape[-1], ValueError,
            f"Input and weight inner dimensions differ: {k} vs {weight.shape[-1]}")
    weight = weight.to(device=x.device)
    col_scale = weight_scale.to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
    require(col_scale.numel() in (1, weight.shape[0]), ValueError,
            "Weight scale must be scalar or per output channel")
    require(rotation_block is None or k % rotation_block == 0, ValueError,
            f"ConvRot group size {rotation_block} does not divide K={k}")
    bias32 = None if bias is None else bias.to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
    return w8a8_linear(x, weight, col_scale, bias32, rotation_block=rotation_block,
                       out_dtype=out_dtype, epilogue="separate")


@contextmanager
def moss_int8_gemm_candidate(*, tile=(32, 64, 64), num_warps=4, num_stages=1, group_m=4,
                             wrapped=False, partial_dot=False):
    """Within the block, Kitchen's eager `int8_linear` export runs the fused
    sm_100a linear: ConvRot and row quantization in the prologue kernel, the
    tcgen05 GEMM with the "separate" fp32 epilogue after it.  Kitchen's
    input-activation and residual helpers still run around it.  Unlike the
    reference (fp32 only), fp16/bf16 inputs and outputs are accelerated;
    other dtypes call the saved export.  Yields hit / fallback statistics."""
    _args.tuning_keywords(tile, num_warps, num_stages, group_m)
    require(wrapped or not partial_dot, ValueError,
            "partial_dot requires the explicitly wrapped-load variant")
    from comfy_kitchen.backends import eager as backend
    from comfy_kitchen.backends.eager import quantization as kitchen_q
    saved_export = backend.int8_linear
    stats = CandidateStats()

    def int8_linear(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16, convrot=False,
                    convrot_groupsize=256, input_act=None, input_act_weight=None, input_act_eps=0.0,
                    residual=None, residual_scale=None):
        if x.dtype not in _args.FLOAT_DTYPES or out_dtype not in _args.FLOAT_DTYPES:
            stats.fallback()
            return saved_export(x, weight, weight_scale, bias=bias, out_dtype=out_dtype, convrot=convrot,
                                convrot_groupsize=convrot_groupsize, input_act=input_act,
                                input_act_weight=input_act_weight, input_act_eps=input_act_eps,
                                residual=residual, residual_scale=residual_scale)
        x = kitchen_q._apply_input_act(x, input_act, input_act_weight, input_act_eps)
        y = _moss_fused_linear(x, weight, weight_scale, bias, out_dtype,
                               convrot_groupsize if convrot else None)
        stats.hit(x.numel() // max(1, x.shape[-1]), weight.shape[0], x.shape[-1])
        return kitchen_q._apply_residual(y, residual, residual_scale)

    with scoped_patch(backend, {"int8_linear": int8_linear}, "MOSS eager export"):
        yield stats


# ------------------------------------------------------------------ Qwen
_QWEN_BRIDGE_SUFFIX = "RDNA2-Qwen21-INT8/rocm_int8_kitchen_patch.py"
# bridge callable -> whether its weight scale is one value per output row
_QWEN_WRAPPERS = (("triton_int8_linear", False), ("triton_int8_linear_per_row", True))


def _loaded_qwen_bridge():
    hits = [mod for mod in list(sys.modules.values())
            if mod is not None and str(getattr(mod, "__file__", "")).endswith(_QWEN_BRIDGE_SUFFIX)]
    require(len(hits) == 1, RuntimeError, "Expected one already-loaded Qwen patientx bridge")
    return hits[0]


def qwen_column_scale(weight_scale, n, device, per_row):
    """The bridge's weight scale as the GEMM's column-scale operand: n
    per-row values for the per-row wrapper; one value (a tensor of any
    shape holding one element, or a Python number) otherwise."""
    if per_row:
        return weight_scale.reshape(n).to(device=device, dtype=torch.float32).contiguous()
    if isinstance(weight_scale, torch.Tensor):
        return weight_scale.to(device=device, dtype=torch.float32, non_blocking=True).reshape(-1).contiguous()
    return torch.full((1,), float(weight_scale), device=device, dtype=torch.float32)


def _qwen_linear(bridge_fn, per_row, stats, gemm_keywords):
    quantize_rows = bridge_fn.__globals__["triton_quantize_rowwise"]

    def linear(x, weight, weight_scale, bias=None, compute_dtype=torch.float16):
        if x.dtype != torch.float32 or compute_dtype != torch.float32:
            stats.fallback()
            return bridge_fn(x, weight, weight_scale, bias=bias, compute_dtype=compute_dtype)
        rows = x.reshape(-1, x.shape[-1])
        codes, row_scale = quantize_rows(rows.float() if per_row else rows)
        col_scale = qwen_column_scale(weight_scale, weight.shape[0], x.device, per_row)
        y = int8_gemm_dequant(codes, weight.T, row_scale.reshape(-1).contiguous(), col_scale, bias,
                              rounding="fused", **gemm_keywords)
        stats.hit(codes.shape[0], weight.shape[0], codes.shape[1])
        return y.reshape(*x.shape[:-1], weight.shape[0])

    return linear


@contextmanager
def qwen_int8_gemm_candidate(patch_module=None, *, tile=(32, 64, 64), num_warps=4, num_stages=1,
                             group_m=4, wrapped=False, partial_dot=False):
    """Within the block, the patientx Qwen bridge's two INT8 GEMM wrappers run
    the sm_100a GEMM with the FMA ("fused") epilogue; the bridge's own row
    quantizer stays in use, and non-fp32 calls go to the saved wrappers.
    The bridge module is found among the loaded modules by its source path
    unless given.  Yields hit / fallback statistics."""
    _args.tuning_keywords(tile, num_warps, num_stages, group_m)
    require(wrapped or not partial_dot, ValueError,
            "partial_dot requires the explicitly wrapped-load variant")
    bridge = patch_module if patch_module is not None else _loaded_qwen_bridge()
    gemm_keywords = dict(tile=tile, num_warps=num_warps, num_stages=num_stages, group_m=group_m,
                         wrapped=wrapped, partial_dot=partial_dot)
    stats = CandidateStats()
    replacements = {name: _qwen_linear(getattr(bridge, name), per_row, stats, gemm_keywords)
                    for name, per_row in _QWEN_WRAPPERS}
    with scoped_patch(bridge, replacements, "Qwen patientx callable"):
        yield stats
