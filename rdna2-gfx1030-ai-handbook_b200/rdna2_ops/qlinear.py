"""B200-native quantized linear: activation prologue + tcgen05 GEMM + epilogue.

Entry points (all enqueue on torch's current stream, allocate only their
outputs and a per-call staging workspace, and never fall back):

  act_quant(x, rotation_block=None, quant="int8")      -> (codes, scale)
  quantize_weight(w, rotation_block=None, quant="int8") -> (codes, scale)
  qgemm(a, w, a_scale, w_scale, bias=None, ...)          -> out
  w8a8_linear(x, w_q, w_scale, bias=None, ...)           -> out
  fp8_linear(x, w_e4m3, w_scale, bias=None, ...)         -> out

Math contract (bit-exact with the CPU oracle):
  rotation  block-Hadamard along K, fp32 butterflies h = 1..B/2 then one
            multiply by fp32(1/sqrt(B)); folded into the weight by rotating
            its rows with the same kernel (H is symmetric and orthonormal).
  quantize  per-row s = absmax/127 (int8) or absmax/448 (e4m3), IEEE
            division, round-half-even, int8 clamp to [-127, 127].
  epilogue  "separate": float(acc)*(sa*sb) + bias in fp32 then one cast
            (rdna2_ops/int8_gemm.py:53-63); "fused": FMA of the same
            (int8_gemm.py:191); "kitchen": cast(float(acc)*(sa*sb)) then + bias
            in the output dtype (production/MOSS_RDNA2_INT8/backend.py:128-143).
"""
from __future__ import annotations

import torch

from . import _args
from . import _native as nat

EPILOGUES = {"separate": nat.EPI_SEPARATE, "fused": nat.EPI_FMA, "kitchen": nat.EPI_KITCHEN}
FLOAT_DTYPES = _args.FLOAT_DTYPES


def set_gemm_path(path):
    """Process-wide GEMM kernel choice: "auto", "single" (1-CTA 128-row
    tiles), "pair" (2-CTA cta_group::2 256-row tiles), or a fixed tile:
    "single256", "single128", "pair256", "pair192", "pair256s" (pair tiles
    with the output staged in shared memory and written by TMA stores; falls
    back to "pair256" for outputs whose rows are not 16-byte aligned),
    "splitk" (M <= 32: swap-AB tiles split along K over a thread-block
    cluster; larger M take "auto"), "pair192s" (256x192 pair tiles with
    TMA stores; "pair192" for unaligned outputs).  INT8 results are bit-identical for every
    choice (floating kinds differ only in fp32 summation order); this is a
    tuning and verification knob."""
    code = {"auto": 0, "single": 1, "pair": 2, "single256": 3, "single128": 4, "pair256": 5,
            "pair192": 6, "pair256s": 7, "splitk": 8, "pair192s": 9}[path]
    nat.check(nat.library().b2_set_gemm_path(code), "b2_set_gemm_path")


def set_prologue_path(path):
    """Process-wide activation-prologue kernel: "auto", "shuffle" (warp
    shuffle butterflies, every quantizer) or "lane" (one lane per 64
    elements, INT8 ties-to-even codes of 16-byte aligned rows; other calls
    fall back to "shuffle").  Codes and scales are bit-identical; this is a
    tuning and verification knob."""
    code = {"auto": 0, "shuffle": 1, "lane": 2}[path]
    nat.check(nat.library().b2_set_prologue_path(code), "b2_set_prologue_path")


def _round_up(v, m):
    return (v + m - 1) // m * m


def _rows_2d(x):
    """View x as [M,K] with unit column stride (copying only if it must)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[-1] > 1 and x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _block(rotation_block, k):
    if rotation_block in (None, 0, 1):
        return 0
    b = int(rotation_block)
    if b & (b - 1) or b > 4096 or k % b:
        raise ValueError(f"Rotation block {b} must be a power of two <= 4096 dividing K={k}")
    return b


def act_quant(x, *, rotation_block=None, quant="int8", out=None, scale=None):
    """Rotate (optionally) and quantize each row of x[..., K].

    Returns (codes [M,K] int8 or float8_e4m3fn, scale [M] fp32), where
    M = prod(x.shape[:-1]).
    """
    if x.dtype not in FLOAT_DTYPES:
        raise TypeError("act_quant expects fp32/fp16/bf16 input")
    if quant not in ("int8", "e4m3"):
        raise ValueError("quant must be 'int8' or 'e4m3'")
    dev = nat.require_device(x)
    x2 = _rows_2d(x)
    m, k = x2.shape
    block = _block(rotation_block, k)
    code_dtype = torch.int8 if quant == "int8" else torch.float8_e4m3fn
    if out is None:
        out = torch.empty((m, k), device=dev, dtype=code_dtype)
    if scale is None:
        scale = torch.empty(m, device=dev, dtype=torch.float32)
    if m == 0:
        return out, scale
    ldx = x2.stride(0) if m > 1 else k
    nat.check(nat.library().b2_act_quant(
        x2.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k, ldx, block, 0 if quant == "int8" else 1,
        out.data_ptr(), out.stride(0) if m > 1 else k, scale.data_ptr(), nat.stream_ptr(dev)),
        "b2_act_quant")
    return out, scale


def quantize_weight(w, *, rotation_block=None, quant="int8"):
    """Per-output-channel quantization of a floating [N,K] weight, with the
    block-Hadamard rotation folded in when rotation_block is set."""
    if w.ndim != 2:
        raise ValueError("Weight must be [N,K]")
    return act_quant(w, rotation_block=rotation_block, quant=quant)


def _operand(t, elem_bytes):
    """(tensor, leading dim) for a [R,K] operand the TMA can read directly,
    or None when the layout needs a repack."""
    r, k = t.shape
    if k > 1 and t.stride(1) != 1:
        return None
    ld = t.stride(0) if r > 1 else _round_up(k, 16 // elem_bytes)
    if ld < k or (ld * elem_bytes) % 16 or t.data_ptr() % 16:
        return None
    return t, ld


def _kmajor(t, elem_bytes, s_row, s_col, rows, cols):
    """Repack an arbitrary strided [rows, cols] view into a padded K-major buffer."""
    ld = _round_up(max(cols, 1), 16 // elem_bytes)
    dtype = torch.uint8 if elem_bytes == 1 else torch.int16
    buf = torch.empty((rows, ld), device=t.device, dtype=dtype)
    nat.check(nat.library().b2_repack(t.data_ptr(), elem_bytes, rows, cols, s_row, s_col,
                                      buf.data_ptr(), ld, nat.stream_ptr(t.device)), "b2_repack")
    return buf, ld


def qgemm_raw(kind, a, w, a_scale, w_scale, bias, epilogue, out):
    """Launch the GEMM on an [M,K] view `a` and an [N,K] view `w` (any strides;
    layouts the TMA cannot read are repacked to K-major first)."""
    m, k = a.shape
    n = w.shape[0]
    eb = 2 if kind in (nat.KIND_BF16, nat.KIND_F16) else 1
    dev = out.device
    if m == 0 or n == 0:
        return out
    if k == 0:
        # Empty reduction: run the kernel over one all-zero k-block.
        a_op = torch.zeros((m, 16 // eb), device=dev, dtype=torch.uint8 if eb == 1 else torch.int16)
        w_op = torch.zeros((n, 16 // eb), device=dev, dtype=a_op.dtype)
        a_t, lda, w_t, ldw, k = a_op, 16 // eb, w_op, 16 // eb, 16 // eb
    else:
        op = _operand(a, eb)
        a_t, lda = op if op else _kmajor(a, eb, a.stride(0), a.stride(1), m, k)
        op = _operand(w, eb)
        w_t, ldw = op if op else _kmajor(w, eb, w.stride(0), w.stride(1), n, k)
    out_code = nat.DTYPE_CODE[out.dtype]
    bias_code = nat.DTYPE_CODE[bias.dtype] if bias is not None else 0
    nat.check(nat.library().b2_qgemm(
        kind, a_t.data_ptr(), lda, w_t.data_ptr(), ldw, m, n, k, nat.ptr(a_scale),
        nat.ptr(w_scale), 0 if w_scale is None else w_scale.numel(), nat.ptr(bias), bias_code,
        epilogue, out.data_ptr(), out_code, out.stride(0) if m > 1 else n,
        nat.stream_ptr(dev)), "b2_qgemm")
    return out


def w8a8_linear(x, w_q, w_scale, bias=None, *, rotation_block=None, out_dtype=None,
                epilogue="separate", kind="int8", workspace=None):
    """y[..., N] = epilogue(quantize(rotate(x)) @ w_q.T) in one C call.

    x fp32/fp16/bf16 [..., K]; w_q int8 (kind "int8") or float8_e4m3fn
    (kind "e4m3") [N,K] as stored; w_scale fp32 [N] or [1]; bias [N] or None.
    """
    if epilogue not in EPILOGUES:
        raise ValueError("epilogue must be one of " + ", ".join(EPILOGUES))
    if x.dtype not in FLOAT_DTYPES:
        raise TypeError("x must be fp32/fp16/bf16")
    want = torch.int8 if kind == "int8" else torch.float8_e4m3fn
    if w_q.dtype != want or w_q.ndim != 2:
        raise TypeError(f"Weight must be a {want} [N,K] tensor")
    dev = nat.require_device(x, w_q, w_scale, bias)
    nat.eager_only(x, bias)
    n, k = w_q.shape
    if x.shape[-1] != k:
        raise ValueError(f"Input and weight inner dimensions must match, got {x.shape[-1]} and {k}")
    _args.fp32_vector(w_scale, n, "w_scale", dev, scalar_ok=True)
    _args.bias_vector(bias, n, dev)
    out_dtype = out_dtype or x.dtype
    x2 = _rows_2d(x)
    m = x2.shape[0]
    out = torch.empty((m, n), device=dev, dtype=out_dtype)
    if m == 0 or n == 0:
        return out.reshape(*x.shape[:-1], n)
    block = _block(rotation_block, k)
    op = _operand(w_q.view(torch.uint8), 1)
    if op is None:
        w_t, ldw = _kmajor(w_q.view(torch.uint8), 1, w_q.stride(0), w_q.stride(1), n, k)
    else:
        w_t, ldw = op
    lib = nat.library()
    need = lib.b2_quant_linear_workspace_bytes(m, k)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=dev, dtype=torch.uint8)
    nat.check(lib.b2_quant_linear(
        nat.KIND_I8 if kind == "int8" else nat.KIND_E4M3, x2.data_ptr(), nat.DTYPE_CODE[x.dtype], m,
        k, x2.stride(0) if m > 1 else k, block, w_t.data_ptr(), ldw, n, w_scale.data_ptr(),
        w_scale.numel(), nat.ptr(bias), nat.DTYPE_CODE[bias.dtype] if bias is not None else 0,
        EPILOGUES[epilogue], out.data_ptr(), nat.DTYPE_CODE[out_dtype], n, workspace.data_ptr(),
        workspace.numel(), nat.stream_ptr(dev)), "b2_quant_linear")
    return out.reshape(*x.shape[:-1], n)


def fp8_linear(x, w_e4m3, w_scale, bias=None, *, out_dtype=None, workspace=None):
    """Scaled FP8 linear: x -> e4m3 with a per-token scale (absmax/448), then
    tcgen05 kind::f8f6f4 against an e4m3 weight with per-channel fp32 scales;
    fp32 accumulation, y = acc*(sa*sw) (+bias), cast to out_dtype (default x's)."""
    return w8a8_linear(x, w_e4m3, w_scale, bias, out_dtype=out_dtype, kind="e4m3",
                       workspace=workspace)
