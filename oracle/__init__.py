"""CPU oracle for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package.  The product (rdna2_ops + the CUDA library)
never calls it.

Thin numpy/ctypes wrapper over qlinear_oracle.c, which restates the reference
math in plain C with IEEE fp32 arithmetic (each C routine cites the reference
file:line it follows).  Storage conventions: fp32 arrays are np.float32; fp16
and bf16 arrays are np.uint16 bit patterns; e4m3 arrays are np.uint8 codes.

Parity pinning: the INT8 GEMM, both epilogues, the INT4 packer and the e4m3
decoder are pinned against golden vectors produced by the reference's own CPU
code (tests/golden/make_golden.py).  The ConvRot rotation and the row
quantizer live in comfy_kitchen 0.2.40, which the reference does not vendor:
for those two the oracle follows the frozen contract in the C header (parity
for them is pinned to that contract, not to reference output).
"""
from __future__ import annotations

import ctypes
import functools

import numpy as np

from .build import build

F32, F16, BF16 = 0, 1, 2
EPI_SEPARATE, EPI_FMA, EPI_KITCHEN = 0, 1, 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int


@functools.lru_cache(maxsize=1)
def lib():
    so = ctypes.CDLL(str(build()))
    sig = {
        "b2o_rotate_rows": [_p, _int, _i64, _i64, _i64, _int, _p],
        "b2o_quant_rows_int8": [_p, _i64, _i64, _p, _i64, _p],
        "b2o_quant_rows_e4m3": [_p, _i64, _i64, _p, _i64, _p],
        "b2o_quant_rows_ref": [_p, _i64, _i64, _p, _i64, _p],
        "b2o_decode_e5m2": [_p, _i64, _p],
        "b2o_gemm_s8": [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _int],
        "b2o_epilogue_s32": [_p, _i64, _p, _p, _i64, _p, _int, _i64, _i64, _int, _p, _int, _i64],
        "b2o_epilogue_f32": [_p, _i64, _p, _p, _p, _int, _i64, _i64, _p, _int, _i64],
        "b2o_w8a8_linear": [_p, _int, _i64, _i64, _i64, _int, _p, _i64, _p, _i64, _p, _int,
                            _i64, _int, _p, _int, _p, _p, _p, _p, _int],
        "b2o_gemm_e4m3_f64": [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _int],
        "b2o_pack_int4": [_p, _i64, _i64, _int, _int, _int, _p, _p, _p, _p],
        "b2o_dequant_int4": [_p, _p, _p, _i64, _i64, _int, _int, _p],
        "b2o_gemm_f32_f64": [_p, _i64, _p, _i64, _i64, _p, _int],
        "b2o_w4a8_linear": [_p, _i64, _i64, _i64, _p, _i64, _p, _int, _p, _p, _int, _p, _p],
        "b2o_encode": [_p, _i64, _int, _p],
        "b2o_decode": [_p, _i64, _int, _p],
        "b2o_encode_e4m3": [_p, _i64, _p],
        "b2o_decode_e4m3": [_p, _i64, _p],
    }
    for name, args in sig.items():
        fn = getattr(so, name)
        fn.argtypes = args
        fn.restype = None
    so.b2o_rotation_scale.argtypes = [_int]
    so.b2o_rotation_scale.restype = ctypes.c_float
    so.b2o_max_threads.restype = _int
    return so


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def max_threads():
    return lib().b2o_max_threads()


# ------------------------------------------------------------------ codecs
def encode(x, dtype):
    """fp32 -> storage bits (RNE).  F32 returns float32, F16/BF16 uint16."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.float32 if dtype == F32 else np.uint16)
    lib().b2o_encode(_ptr(x), x.size, dtype, _ptr(out))
    return out


def decode(bits, dtype):
    bits = _c(bits, np.float32 if dtype == F32 else np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().b2o_decode(_ptr(bits), bits.size, dtype, _ptr(out))
    return out


def encode_e4m3(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().b2o_encode_e4m3(_ptr(x), x.size, _ptr(out))
    return out


def decode_e4m3(codes):
    codes = _c(codes, np.uint8)
    out = np.empty(codes.shape, np.float32)
    lib().b2o_decode_e4m3(_ptr(codes), codes.size, _ptr(out))
    return out


# ---------------------------------------------------------------- prologue
def rotation_scale(block):
    return float(lib().b2o_rotation_scale(block))


def rotate_rows(x, dtype, block):
    """x: [M,K] storage array of `dtype`; block 0/1 = no rotation -> fp32."""
    x = _c(x, np.float32 if dtype == F32 else np.uint16)
    m, k = x.shape
    out = np.empty((m, k), np.float32)
    lib().b2o_rotate_rows(_ptr(x), dtype, m, k, k, int(block or 0), _ptr(out))
    return out


def quant_rows_int8(xf):
    xf = _c(xf, np.float32)
    m, k = xf.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().b2o_quant_rows_int8(_ptr(xf), m, k, _ptr(q), k, _ptr(s))
    return q, s


def quant_rows_e4m3(xf):
    xf = _c(xf, np.float32)
    m, k = xf.shape
    q = np.empty((m, k), np.uint8)
    s = np.empty(m, np.float32)
    lib().b2o_quant_rows_e4m3(_ptr(xf), m, k, _ptr(q), k, _ptr(s))
    return q, s


def quant_rows_ref(xf):
    """The reference's _quant_rows (fp8_weight_gemm_v06.py:76-92)."""
    xf = _c(xf, np.float32)
    m, k = xf.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().b2o_quant_rows_ref(_ptr(xf), m, k, _ptr(q), k, _ptr(s))
    return q, s


def decode_e5m2(codes):
    codes = _c(codes, np.uint8)
    out = np.empty(codes.shape, np.float32)
    lib().b2o_decode_e5m2(_ptr(codes), codes.size, _ptr(out))
    return out


def act_quant_int8(x, dtype, block):
    return quant_rows_int8(rotate_rows(x, dtype, block))


# -------------------------------------------------------------------- GEMM
def gemm_s8(a, w, threads=0):
    """a int8 [M,K], w int8 [N,K] -> exact int32 [M,N]."""
    a = _c(a, np.int8)
    w = _c(w, np.int8)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), np.int32)
    lib().b2o_gemm_s8(_ptr(a), k, _ptr(w), k, m, n, k, _ptr(c), n, int(threads))
    return c


def epilogue_s32(acc, sa, sb, bias=None, bias_dtype=F32, mode=EPI_SEPARATE, out_dtype=F32):
    acc = _c(acc, np.int32)
    m, n = acc.shape
    sa = _c(sa, np.float32).reshape(-1)
    sb = _c(sb, np.float32).reshape(-1)
    if bias is not None:
        bias = _c(bias, np.float32 if bias_dtype == F32 else np.uint16).reshape(-1)
    out = np.empty((m, n), np.float32 if out_dtype == F32 else np.uint16)
    lib().b2o_epilogue_s32(_ptr(acc), n, _ptr(sa), _ptr(sb), sb.size, _ptr(bias), bias_dtype,
                           m, n, mode, _ptr(out), out_dtype, n)
    return out


def w8a8_linear(x, x_dtype, block, w, sw, bias=None, bias_dtype=F32, mode=EPI_SEPARATE,
                out_dtype=F16, threads=0):
    """Whole fused linear on the CPU: rotate+quantize x, exact GEMM, epilogue."""
    x = _c(x, np.float32 if x_dtype == F32 else np.uint16)
    w = _c(w, np.int8)
    m, k = x.shape
    n = w.shape[0]
    sw = _c(sw, np.float32).reshape(-1)
    if bias is not None:
        bias = _c(bias, np.float32 if bias_dtype == F32 else np.uint16).reshape(-1)
    out = np.empty((m, n), np.float32 if out_dtype == F32 else np.uint16)
    xr = np.empty((m, k), np.float32)
    q = np.empty((m, k), np.int8)
    sa = np.empty(m, np.float32)
    acc = np.empty((m, n), np.int32)
    lib().b2o_w8a8_linear(_ptr(x), x_dtype, m, k, k, int(block or 0), _ptr(w), k, _ptr(sw),
                          sw.size, _ptr(bias), bias_dtype, n, mode, _ptr(out), out_dtype,
                          _ptr(xr), _ptr(q), _ptr(sa), _ptr(acc), int(threads))
    return out


def gemm_e4m3_f64(a, w, threads=0):
    a = _c(a, np.uint8)
    w = _c(w, np.uint8)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), np.float64)
    lib().b2o_gemm_e4m3_f64(_ptr(a), k, _ptr(w), k, m, n, k, _ptr(c), int(threads))
    return c


def epilogue_f32(acc, sa, sb, bias=None, bias_dtype=F32, out_dtype=BF16):
    acc = _c(acc, np.float64)
    m, n = acc.shape
    sa = _c(sa, np.float32).reshape(-1)
    sb = _c(sb, np.float32).reshape(-1)
    if bias is not None:
        bias = _c(bias, np.float32 if bias_dtype == F32 else np.uint16).reshape(-1)
    out = np.empty((m, n), np.float32 if out_dtype == F32 else np.uint16)
    lib().b2o_epilogue_f32(_ptr(acc), n, _ptr(sa), _ptr(sb), _ptr(bias), bias_dtype, m, n,
                           _ptr(out), out_dtype, n)
    return out


# -------------------------------------------------------------------- INT4
def pack_int4(w, group_size=128, symmetric=False, order="low"):
    """Restatement of pack_int4_cpu for layout "nk" -> dict of arrays."""
    w = _c(w, np.float32)
    n, k = w.shape
    g = k // group_size
    data = np.empty((n, k // 8), np.int32)
    scales = np.empty((n, g), np.float32)
    zeros = np.empty((n, g), np.int32)
    sums = np.empty((n, g), np.int32)
    lib().b2o_pack_int4(_ptr(w), n, k, group_size, int(bool(symmetric)), int(order == "high"),
                        _ptr(data), _ptr(scales), _ptr(zeros), _ptr(sums))
    return {"data": data, "scales": scales, "zeros": zeros, "sums": sums}


def dequant_int4(words, scales, zeros, group_size, out_dtype=BF16):
    """Signed-nibble words (order low) -> fp32 values rounded through out_dtype."""
    words = _c(words, np.int32)
    n, k8 = words.shape
    k = k8 * 8
    scales = _c(scales, np.float32)
    zeros = _c(zeros, np.float32)
    out = np.empty((n, k), np.float32)
    lib().b2o_dequant_int4(_ptr(words), _ptr(scales), _ptr(zeros), n, k, group_size, out_dtype,
                           _ptr(out))
    return out


def gemm_f32_f64(a, w, threads=0):
    a = _c(a, np.float32)
    w = _c(w, np.float32)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), np.float64)
    lib().b2o_gemm_f32_f64(_ptr(a), m, _ptr(w), n, k, _ptr(c), int(threads))
    return c


def w4a8_linear(a8, centered, scales, group, sa, bias=None, integer=False):
    """W4A8 grouped linear (reference grouped_integer_reference order):
    a8 int8 [M,K], centered int8 [N,K] (= q - z), scales fp32 [N, K/group],
    sa fp32 [M], bias fp32 [N] or None -> fp32 [M,N] (int32 when integer)."""
    a8 = _c(a8, np.int8)
    centered = _c(centered, np.int8)
    scales = _c(scales, np.float32)
    sa = _c(np.asarray(sa).reshape(-1), np.float32)
    m, k = a8.shape
    n = centered.shape[0]
    b = None if bias is None else _c(np.asarray(bias).reshape(-1), np.float32)
    out_f = np.zeros((m, n), np.float32)
    out_i = np.zeros((m, n), np.int32)
    lib().b2o_w4a8_linear(_ptr(a8), k, m, k, _ptr(centered), n, _ptr(scales), int(group), _ptr(sa),
                          _ptr(b), int(bool(integer)), _ptr(out_f), _ptr(out_i))
    return out_i if integer else out_f
