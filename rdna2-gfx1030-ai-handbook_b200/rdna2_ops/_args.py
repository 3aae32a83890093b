"""Argument checks shared by every operator module of this package.

Each check raises the exception class the reference raises for the same
mistake (ValueError for shape / device / stride / layout problems, TypeError
for wrong dtypes or non-tensors, RuntimeError for calls outside explicit
eager mode), so callers written against the reference keep working.  The
checks themselves are stated as small predicates over the tensors; the
operator modules compose them instead of restating them.
"""
from __future__ import annotations

import torch

from . import _native as nat

FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)

# |sum_k a*b| <= K * 127 * 128 must stay below 2**31 for any signed INT8 operands
# (-128 * -128 included): K <= 131071.
INT32_SAFE_K = (2 ** 31 - 1) // (128 * 128)


def require(ok, exc, message):
    if not ok:
        raise exc(message)


def int8_operands(a, b):
    """a [M,K] and b [K,N], both int8, on one sm_100 device, non-negative
    strides, K small enough that the INT32 accumulator cannot overflow.
    Returns (M, N, K, device)."""
    require(a.ndim == 2 and b.ndim == 2 and a.shape[1] == b.shape[0], ValueError,
            f"Expected [M,K] @ [K,N] operands, got {tuple(a.shape)} and {tuple(b.shape)}")
    require(a.dtype == torch.int8 and b.dtype == torch.int8, TypeError,
            f"INT8 GEMM operands must both be int8, got {a.dtype} and {b.dtype}")
    require(a.device.type == "cuda" and b.device == a.device, ValueError,
            "GEMM operands must live on one CUDA device")
    dev = nat.require_device(a, b)
    require(min(a.stride() + b.stride()) >= 0, ValueError, "Negative strides are unsupported")
    require(a.shape[1] <= INT32_SAFE_K, ValueError,
            f"K={a.shape[1]} exceeds {INT32_SAFE_K}: the INT32 accumulator could overflow")
    return a.shape[0], b.shape[1], a.shape[1], dev


def tuning_keywords(tile, num_warps, num_stages, group_m):
    """The reference's Triton launch keywords.  They are checked for the same
    domains the reference accepts and otherwise unused: the sm_100a kernels
    choose their own persistent tiles."""
    require(len(tile) == 3 and all(16 <= v <= 256 and v & (v - 1) == 0 for v in tile), ValueError,
            f"tile must be three powers of two in [16, 256], got {tuple(tile)}")
    require(num_warps in (4, 8) and num_stages in (1, 2, 3) and group_m in (1, 2, 4, 8), ValueError,
            f"Unsupported launch configuration num_warps={num_warps} num_stages={num_stages} "
            f"group_m={group_m}")


def eager_call():
    require(not (torch.compiler.is_compiling() or torch.cuda.is_current_stream_capturing()),
            RuntimeError, "Only explicit eager calls are supported")


def no_autograd(*tensors):
    require(not (torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)),
            ValueError, "Autograd is unsupported")


def fp32_vector(t, length, label, device, scalar_ok=False):
    """A contiguous fp32 device vector of `length` elements (or one element
    when scalar_ok)."""
    require(isinstance(t, torch.Tensor), TypeError, f"{label} must be a device tensor")
    require(t.device == device and t.dtype == torch.float32 and t.is_contiguous(), ValueError,
            f"{label} must be contiguous fp32 on {device}")
    require(t.numel() == length or (scalar_ok and t.numel() == 1), ValueError,
            f"{label} has {t.numel()} elements, expected {length}" + (" or 1" if scalar_ok else ""))


def bias_vector(bias, length, device):
    if bias is None:
        return
    require(isinstance(bias, torch.Tensor) and bias.device == device and bias.numel() == length
            and bias.is_contiguous() and bias.dtype in FLOAT_DTYPES, ValueError,
            f"bias must be a contiguous fp32/fp16/bf16 vector of length {length} on {device}")


def output_dtype(dtype):
    require(dtype in FLOAT_DTYPES, TypeError, f"out_dtype must be fp32, fp16 or bf16, got {dtype}")
