"""INT8 GEMM with an optional fused FP32 dequantization epilogue, on sm_100a.

Drop-in for the reference module rdna2_ops/int8_gemm.py (same public names
and signatures).  The contraction runs on tcgen05 kind::i8 tensor cores with
TMEM accumulators (csrc/qgemm.cu) instead of the gfx1030 dot4 Triton kernels
_int8_dot_dequant / _int8_dot_dequant_wrapped (int8_gemm.py:19-123).

Kept from the reference contract:
  * the scale order float(acc) * (row_scale * col_scale) (int8_gemm.py:53-63);
  * rounding="separate" forbids multiply/add contraction, rounding="fused"
    uses one FMA (int8_gemm.py:191);
  * B is read through its strides, so weight.T needs no copy
    (int8_gemm.py:39-40); other layouts are repacked once per call;
  * validation and eager-only policy (int8_gemm.py:131-149);
  * a fresh output per call (int8_gemm.py:178).
Tile / warp / stage / group_m keywords are validated like the reference and
otherwise ignored: the B200 kernel sizes its own persistent tiles.
Extension: `out_dtype` (fp32 default) lets the epilogue cast straight to
fp16/bf16.
"""
from contextlib import contextmanager
import sys

import torch

from . import _native as nat
from .qlinear import act_quant, qgemm_raw

_K_MAX = 131071


def _validate(a, b, tile, num_warps, num_stages, group_m):
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("Expected [M,K] @ [K,N]")
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise TypeError("Both GEMM operands must be INT8")
    if a.device.type != "cuda" or b.device != a.device:
        raise ValueError("Inputs must share a CUDA device")
    nat.require_device(a, b)
    if any(s < 0 for s in a.stride() + b.stride()):
        raise ValueError("Negative strides are unsupported")
    if a.shape[1] > _K_MAX:
        raise ValueError("K could overflow signed INT32 for arbitrary signed INT8 inputs")
    if len(tile) != 3 or any(v < 16 or v > 256 or v & (v - 1) for v in tile):
        raise ValueError("Tile dimensions must be powers of two in [16,256]")
    if num_warps not in (4, 8) or num_stages not in (1, 2, 3) or group_m not in (1, 2, 4, 8):
        raise ValueError("Unsupported launch configuration")
    if torch.compiler.is_compiling() or torch.cuda.is_current_stream_capturing():
        raise RuntimeError("Only explicit eager calls are supported")


def _launch(a, b, a_scale, b_scale, bias, *, tile, num_warps, num_stages, group_m, rounding,
            return_kernel, wrapped=False, partial_dot=False, out_dtype=torch.float32):
    _validate(a, b, tile, num_warps, num_stages, group_m)
    if partial_dot and not wrapped:
        raise ValueError("partial_dot requires the explicitly wrapped-load variant")
    dequant = a_scale is not None
    m, k = a.shape
    n = b.shape[1]
    if rounding not in ("separate", "fused"):
        raise ValueError("rounding must be separate or fused")
    if dequant:
        for value, size, label in ((a_scale, m, "a_scale"), (b_scale, n, "b_scale")):
            if not isinstance(value, torch.Tensor):
                raise TypeError(label + " must be a device tensor")
            if value.device != a.device or value.dtype != torch.float32 or not value.is_contiguous():
                raise ValueError(label + " must be contiguous FP32 on the input device")
            if value.numel() != size and not (label == "b_scale" and value.numel() == 1):
                raise ValueError(label + " has the wrong number of elements")
            if torch.is_grad_enabled() and value.requires_grad:
                raise ValueError("Autograd is unsupported")
        if bias is not None:
            if (bias.device != a.device or bias.numel() != n or not bias.is_contiguous()
                    or bias.dtype not in (torch.float32, torch.float16, torch.bfloat16)):
                raise ValueError("Bias must be a contiguous floating point vector of length N")
            if torch.is_grad_enabled() and bias.requires_grad:
                raise ValueError("Autograd is unsupported")
        if out_dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise TypeError("out_dtype must be fp32, fp16 or bf16")
    out = torch.empty((m, n), device=a.device, dtype=out_dtype if dequant else torch.int32)
    if m == 0 or n == 0:
        return (out, None) if return_kernel else out
    epilogue = (nat.EPI_SEPARATE if rounding == "separate" else nat.EPI_FMA) if dequant else nat.EPI_NONE
    qgemm_raw(nat.KIND_I8, a, b.T, a_scale if dequant else None, b_scale if dequant else None,
              bias if dequant else None, epilogue, out)
    kernel = {"name": "qgemm_kernel<kind::i8>", "arch": "sm_100a"} if return_kernel else None
    return (out, kernel) if return_kernel else out


def int8_matmul(a, b, *, tile=(32, 64, 64), num_warps=4, num_stages=1,
                group_m=4, return_kernel=False, wrapped=False, partial_dot=False):
    """Exact INT8 -> INT32 matmul; accepts both [K,N] layouts without copying
    the weight.T view (reference int8_gemm.py:195-200)."""
    return _launch(a, b, None, None, None, tile=tile, num_warps=num_warps,
                   num_stages=num_stages, group_m=group_m, rounding="separate",
                   return_kernel=return_kernel, wrapped=wrapped, partial_dot=partial_dot)


def int8_gemm_dequant(a, b, a_scale, b_scale, bias=None, *, tile=(32, 64, 64),
                      num_warps=4, num_stages=1, group_m=4,
                      rounding="separate", return_kernel=False, wrapped=False, partial_dot=False,
                      out_dtype=torch.float32):
    """INT32 GEMM and row/scalar or row/column FP32 dequantization in one kernel
    (reference int8_gemm.py:203-214).  Inputs are already quantized; a fresh
    output is allocated.  Finite scales/bias are a precondition."""
    return _launch(a, b, a_scale, b_scale, bias, tile=tile, num_warps=num_warps,
                   num_stages=num_stages, group_m=group_m, rounding=rounding,
                   return_kernel=return_kernel, wrapped=wrapped, partial_dot=partial_dot,
                   out_dtype=out_dtype)


@contextmanager
def moss_int8_gemm_candidate(*, tile=(32, 64, 64), num_warps=4, num_stages=1, group_m=4,
                             wrapped=False, partial_dot=False):
    """Scoped replacement of Kitchen's eager int8_linear export (reference
    int8_gemm.py:217-271).  Kitchen's input activation and residual helpers
    are preserved; ConvRot + row quantization run in the fused sm_100a
    prologue and the GEMM + "separate" epilogue in the tcgen05 kernel.
    Unlike the reference, fp16/bf16 calls are accelerated too (the epilogue
    casts to out_dtype); only unsupported shapes fall back to the saved export.
    """
    from comfy_kitchen.backends import eager as backend
    from comfy_kitchen.backends.eager import quantization as q
    original = backend.int8_linear
    stats = {"hits": 0, "fallbacks": 0, "shapes": {}}

    def candidate(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16,
                  convrot=False, convrot_groupsize=256, input_act=None,
                  input_act_weight=None, input_act_eps=0.0,
                  residual=None, residual_scale=None):
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16) or out_dtype not in (
                torch.float32, torch.float16, torch.bfloat16):
            stats["fallbacks"] += 1
            return original(x, weight, weight_scale, bias=bias, out_dtype=out_dtype,
                            convrot=convrot, convrot_groupsize=convrot_groupsize,
                            input_act=input_act, input_act_weight=input_act_weight,
                            input_act_eps=input_act_eps, residual=residual,
                            residual_scale=residual_scale)
        x = q._apply_input_act(x, input_act, input_act_weight, input_act_eps)
        if x.shape[-1] != weight.shape[-1]:
            raise ValueError("Input and weight inner dimensions differ")
        weight = weight.to(device=x.device)
        ws = weight_scale.to(device=x.device, dtype=torch.float32).reshape(-1)
        if ws.numel() not in (1, weight.shape[0]):
            raise ValueError("Weight scale must be scalar or per output channel")
        if convrot and x.shape[-1] % convrot_groupsize:
            raise ValueError("ConvRot group size does not divide K")
        shape = x.shape
        a, sa = act_quant(x.reshape(-1, shape[-1]),
                          rotation_block=convrot_groupsize if convrot else None)
        bias32 = None if bias is None else bias.to(device=x.device, dtype=torch.float32).reshape(-1)
        y = int8_gemm_dequant(a, weight.T, sa, ws.contiguous(), bias32, tile=tile,
                              num_warps=num_warps, num_stages=num_stages, group_m=group_m,
                              rounding="separate", wrapped=wrapped, partial_dot=partial_dot,
                              out_dtype=out_dtype)
        stats["hits"] += 1
        key = str((a.shape[0], weight.shape[0], a.shape[1]))
        stats["shapes"][key] = stats["shapes"].get(key, 0) + 1
        return q._apply_residual(y.reshape(*shape[:-1], weight.shape[0]), residual, residual_scale)

    backend.int8_linear = candidate
    try:
        yield stats
    finally:
        if backend.int8_linear is not candidate:
            raise RuntimeError("MOSS eager export changed during the research context")
        backend.int8_linear = original


@contextmanager
def qwen_int8_gemm_candidate(patch_module=None, *, tile=(32, 64, 64), num_warps=4, num_stages=1,
                             group_m=4, wrapped=False, partial_dot=False):
    """Scoped replacement of the patientx bridge's two GEMM wrappers (reference
    int8_gemm.py:274-330): the bridge's own row quantizer stays in use, the
    GEMM + FMA ("fused") epilogue runs on the sm_100a kernel."""
    if patch_module is None:
        found = [m for m in tuple(sys.modules.values()) if m is not None
                 and str(getattr(m, "__file__", "")).endswith(
                     "RDNA2-Qwen21-INT8/rocm_int8_kitchen_patch.py")]
        if len(found) != 1:
            raise RuntimeError("Expected one already-loaded Qwen patientx bridge")
        patch_module = found[0]
    names = ("triton_int8_linear", "triton_int8_linear_per_row")
    originals = {name: getattr(patch_module, name) for name in names}
    stats = {"hits": 0, "fallbacks": 0, "shapes": {}}
    replacements = {}

    def make_wrapper(original, per_row):
        quantize = original.__globals__["triton_quantize_rowwise"]

        def candidate(x, weight, weight_scale, bias=None, compute_dtype=torch.float16):
            if x.dtype != torch.float32 or compute_dtype != torch.float32:
                stats["fallbacks"] += 1
                return original(x, weight, weight_scale, bias=bias, compute_dtype=compute_dtype)
            shape = x.shape
            x2d = x.reshape(-1, shape[-1])
            a, sa = quantize(x2d.float() if per_row else x2d)
            if per_row:
                ws = weight_scale.reshape(weight.shape[0]).contiguous()
            elif isinstance(weight_scale, torch.Tensor):
                ws = weight_scale.to(x.device, non_blocking=True).reshape(-1)
            else:
                ws = torch.tensor([weight_scale], device=x.device, dtype=torch.float32)
            y = int8_gemm_dequant(a, weight.T, sa.reshape(-1).contiguous(), ws, bias, tile=tile,
                                  num_warps=num_warps, num_stages=num_stages, group_m=group_m,
                                  rounding="fused", wrapped=wrapped, partial_dot=partial_dot)
            stats["hits"] += 1
            key = str((a.shape[0], weight.shape[0], a.shape[1]))
            stats["shapes"][key] = stats["shapes"].get(key, 0) + 1
            return y.reshape(*shape[:-1], weight.shape[0])
        return candidate

    for name, original in originals.items():
        replacements[name] = make_wrapper(original, name.endswith("per_row"))
        setattr(patch_module, name, replacements[name])
    try:
        yield stats
    finally:
        for name in names:
            if getattr(patch_module, name) is not replacements[name]:
                raise RuntimeError("Qwen patientx callable changed during the research context")
        for name, original in originals.items():
            setattr(patch_module, name, original)
