"""Group-quantized INT4 weight GEMM on sm_100a (drop-in for the reference's
rdna2_ops/int4_weight_gemm_v07.py).

Storage contract kept from the reference (int4_weight_gemm_v07.py:1-46):
linear INT4, W = (q - zero) * scale per output row and K group, caller-owned
packs, no hidden cache.  `PackedInt4` keeps the reference's fields and
encodings (signed nibbles q, fp32 scales, int32 zeros = zu - 8, int32 sums,
layouts "nk"/"kn", nibble orders "low"/"high").

The B200 kernel (csrc/w4a16.cu) reads uint4 weights with 16-bit scales and
zero points zu in the activation dtype, stored as 4 KiB (128-row x 64-K)
tiles so that each CTA streams one contiguous byte range.  `prepare_w4a16`
builds that caller-owned `W4A16Weight` from a PackedInt4 on the device (the
nibble flip u = q + 8 and zu = z + 8 are lossless; the scale cast to 16 bits
is the one rounding).  `int4_linear_a16` accepts either; a PackedInt4 is
converted per call.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from .convrot_checkpoint import check_current, source_stamp
from .qlinear import qgemm_raw

_GROUPS = (32, 64, 128)


@dataclass
class PackedInt4:
    data: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    sums: torch.Tensor
    n: int
    k: int
    group_size: int
    symmetric: bool
    layout: str = "nk"
    order: str = "low"

    def to(self, device):
        return PackedInt4(*(t.to(device) for t in (self.data, self.scales, self.zeros, self.sums)),
                          self.n, self.k, self.group_size, self.symmetric, self.layout, self.order)

    @property
    def bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.data, self.scales, self.zeros, self.sums))

    @property
    def logical_stride(self):
        return self.data.stride() if self.layout == "nk" else self.data.T.stride()


@dataclass
class W4A16Weight:
    """B200 weight format (include/b2_qlinear.h, b2_w4a16_prepare):
    `tiles` int32 [T, K/64, 128, 8] with T = ceil(N/128) -- unsigned nibbles,
    element j = k % 8 of a word at nibble (j >> 1) + 4*(j & 1); `groups`
    int32 [T, K/group, 128] -- low half the scale, high half the zero point
    zu, both in `dtype`.  Rows past N are zero.  `source` stamps the
    PackedInt4 it was prepared from (convrot_checkpoint.source_stamp)."""
    tiles: torch.Tensor
    groups: torch.Tensor
    n: int
    k: int
    group_size: int
    dtype: torch.dtype
    source: tuple | None = None

    @property
    def bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.tiles, self.groups))

    def clone(self):
        return W4A16Weight(self.tiles.clone(), self.groups.clone(), self.n, self.k, self.group_size,
                           self.dtype, self.source)

    def is_current(self, p):
        """False once PackedInt4 `p` changed since this pack was prepared."""
        return self.source is None or self.source == source_stamp(p)


@dataclass
class W4A8Weight:
    """B200 W4A8 format (include/b2_qlinear.h, b2_w4a8_prepare): `tiles`
    uint8 bytes of u64 [T, K/128, 8, 128] unsigned nibbles in the int8-unpack
    order; `groups` u64 [T, K/group, 128] = {fp32 scale, zu}.  `source`
    stamps the PackedInt4 it was prepared from."""
    tiles: torch.Tensor
    groups: torch.Tensor
    n: int
    k: int
    group_size: int
    source: tuple | None = None

    @property
    def bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.tiles, self.groups))

    def is_current(self, p):
        """False once PackedInt4 `p` changed since this pack was prepared."""
        return self.source is None or self.source == source_stamp(p)


# ------------------------------------------------------------ CPU packer
def pack_int4_cpu(w, *, group_size=64, symmetric=True, layout="nk", order="low"):
    """Independent CPU packer (reference int4_weight_gemm_v07.py:49-82):
    ties-to-even rounding, explicit ranges, zero groups -> scale 1, q = z = 0."""
    if w.device.type != "cpu" or w.ndim != 2 or not w.is_floating_point():
        raise ValueError("CPU floating-point [N,K] weight required")
    n, k = w.shape
    if group_size not in _GROUPS or k % group_size or layout not in ("nk", "kn") or order not in ("low", "high"):
        raise ValueError("K must be divisible by group size 32/64/128; valid layout/order required")
    if not torch.isfinite(w).all():
        raise ValueError("Finite weight required")
    x = w.float().reshape(n, k // group_size, group_size)
    if symmetric:
        scales = x.abs().amax(-1) / 7
        scales = torch.where(scales == 0, torch.ones_like(scales), scales)
        zeros = torch.zeros_like(scales, dtype=torch.int32)
        q = torch.round(x / scales[..., None]).clamp(-7, 7).to(torch.int32)
    else:
        lo = torch.clamp(x.amin(-1), max=0.0)
        hi = torch.clamp(x.amax(-1), min=0.0)
        scales = (hi - lo) / 15
        empty = scales == 0
        scales = torch.where(empty, torch.ones_like(scales), scales)
        zu = torch.round(-lo / scales).clamp(0, 15).to(torch.int32)
        zeros = torch.where(empty, torch.zeros_like(zu), zu - 8)
        q = (torch.round(x / scales[..., None]) + zu[..., None]).clamp(0, 15).to(torch.int32) - 8
        q = torch.where(empty[..., None], torch.zeros_like(q), q)
    sums = q.sum(-1, dtype=torch.int32)
    nib = q.reshape(n, k // 8, 8).to(torch.int64) & 15
    shifts = torch.arange(8, dtype=torch.int64) * 4
    if order == "high":
        shifts = 28 - shifts
    words = (nib << shifts).sum(-1).to(torch.int32)
    if layout == "kn":
        words = words.T.contiguous()
    return PackedInt4(words, scales.contiguous(), zeros.contiguous(), sums.contiguous(), n, k,
                      group_size, bool(symmetric), layout, order)


def unpack_int4_cpu(p, *, floating=True):
    """CPU decode (reference int4_weight_gemm_v07.py:85-92): q - z, or (q - z) * s."""
    words = p.data.cpu() if p.layout == "nk" else p.data.cpu().T
    shifts = torch.arange(8, dtype=torch.int64) * 4
    if p.order == "high":
        shifts = 28 - shifts
    q = ((words.to(torch.int64)[..., None] >> shifts) & 15).to(torch.int32)
    q = torch.where(q >= 8, q - 16, q).reshape(p.n, p.k // p.group_size, p.group_size)
    centered = q - p.zeros.cpu()[..., None]
    if not floating:
        return centered.reshape(p.n, p.k)
    return (centered.float() * p.scales.cpu()[..., None]).reshape(p.n, p.k)


# --------------------------------------------------------- GPU pack/unpack
def _validate(p):
    if not isinstance(p, PackedInt4) or p.data.device.type != "cuda":
        raise ValueError("PackedInt4 on a CUDA device required")
    nat.require_device(p.data)
    if (p.group_size not in _GROUPS or min(p.n, p.k) <= 0 or p.k % p.group_size or p.n * p.k >= 2**31
            or p.layout not in ("nk", "kn") or p.order not in ("low", "high")
            or p.data.dtype != torch.int32 or not p.data.is_contiguous()
            or tuple(p.data.shape) != ((p.n, p.k // 8) if p.layout == "nk" else (p.k // 8, p.n))):
        raise ValueError("Invalid packed shape/storage")
    for t, dtype in ((p.scales, torch.float32), (p.zeros, torch.int32), (p.sums, torch.int32)):
        if (t.device != p.data.device or t.dtype != dtype or tuple(t.shape) != (p.n, p.k // p.group_size)
                or not t.is_contiguous()):
            raise ValueError("Invalid scale/zero/sum storage")
    nat.eager_only(p.data, p.scales)


def pack_int4(w, *, group_size=64, symmetric=True, layout="nk", order="low"):
    """Device packer with pack_int4_cpu's exact semantics (csrc/w4a16.cu)."""
    if w.ndim != 2 or not w.is_floating_point() or w.dtype not in nat.DTYPE_CODE:
        raise ValueError("Floating [N,K] weight required")
    dev = nat.require_device(w)
    nat.eager_only(w)
    n, k = w.shape
    if group_size not in _GROUPS or k % group_size or min(n, k) <= 0 or n * k >= 2**31:
        raise ValueError("Nonempty bounded shape and K divisible by 32/64/128 required")
    if layout not in ("nk", "kn") or order not in ("low", "high"):
        raise ValueError("Unknown packing layout/order")
    if w.stride(1) != 1:
        w = w.contiguous()
    data = torch.empty((n, k // 8) if layout == "nk" else (k // 8, n), device=dev, dtype=torch.int32)
    scales = torch.empty((n, k // group_size), device=dev, dtype=torch.float32)
    zeros = torch.empty_like(scales, dtype=torch.int32)
    sums = torch.empty_like(zeros)
    nat.check(nat.library().b2_pack_int4(
        w.data_ptr(), nat.DTYPE_CODE[w.dtype], w.stride(0) if n > 1 else k, n, k, group_size,
        int(bool(symmetric)), int(layout == "kn"), int(order == "high"), data.data_ptr(),
        scales.data_ptr(), zeros.data_ptr(), sums.data_ptr(), nat.stream_ptr(dev)), "b2_pack_int4")
    return PackedInt4(data, scales, zeros, sums, n, k, group_size, bool(symmetric), layout, order)


def unpack_int4(p, *, dtype=torch.float16):
    """Device decode: (q - z) * s as fp16/fp32, or the integer q - z as int8."""
    _validate(p)
    if dtype not in (torch.float16, torch.float32, torch.int8):
        raise TypeError(dtype)
    out = torch.empty((p.n, p.k), device=p.data.device, dtype=dtype)
    code = {torch.float32: nat.F32, torch.float16: nat.F16, torch.int8: 3}[dtype]
    nat.check(nat.library().b2_unpack_int4(
        p.data.data_ptr(), int(p.layout == "kn"), int(p.order == "high"), p.scales.data_ptr(),
        p.zeros.data_ptr(), p.n, p.k, p.group_size, code, out.data_ptr(),
        nat.stream_ptr(p.data.device)), "b2_unpack_int4")
    return out


def prepare_w4a16(p, dtype=torch.bfloat16):
    """Caller-owned B200 weight: unsigned nibbles, 16-bit scales/zero points."""
    _validate(p)
    if dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("W4A16 weights pair with fp16 or bf16 activations")
    if p.k % 64:
        raise ValueError("W4A16 kernel needs K divisible by 64")
    lib = nat.library()
    t = -(-p.n // 128)
    tiles = torch.empty((t, p.k // 64, 128, 8), device=p.data.device, dtype=torch.int32)
    groups = torch.empty((t, p.k // p.group_size, 128), device=p.data.device, dtype=torch.int32)
    assert tiles.numel() * 4 == lib.b2_w4a16_tiles_bytes(p.n, p.k)
    assert groups.numel() * 4 == lib.b2_w4a16_groups_bytes(p.n, p.k, p.group_size)
    nat.check(lib.b2_w4a16_prepare(
        p.data.data_ptr(), int(p.layout == "kn"), int(p.order == "high"), p.scales.data_ptr(),
        p.zeros.data_ptr(), p.n, p.k, p.group_size, nat.DTYPE_CODE[dtype], tiles.data_ptr(),
        groups.data_ptr(), nat.stream_ptr(p.data.device)), "b2_w4a16_prepare")
    return W4A16Weight(tiles, groups, p.n, p.k, p.group_size, dtype, source_stamp(p))


def quantize_w4a16(w, *, group_size=128, dtype=torch.bfloat16):
    """Affine uint4 group quantization (zero point per group) straight to the
    B200 format: pack_int4(symmetric=False) then prepare_w4a16."""
    return prepare_w4a16(pack_int4(w, group_size=group_size, symmetric=False), dtype)


def set_w4a16_path(path):
    """Process-wide W4A16 decode kernel for M <= 32: "auto", "smem" (the
    dequantized weights staged in shared memory) or "tmem" (kept in tensor
    memory as the MMA's A operand).  Both dequantize identically; outputs
    differ only in the tensor core's fp32 summation order.  A tuning and
    verification knob."""
    code = {"auto": 0, "smem": 1, "tmem": 2}[path]
    nat.check(nat.library().b2_set_w4a16_path(code), "b2_set_w4a16_path")


def w4a16_gemm(a, wt, bias=None, *, workspace=None):
    """y = a @ dequant(wt).T (+ bias) on the tcgen05 W4A16 kernel."""
    if not isinstance(wt, W4A16Weight):
        raise TypeError("W4A16Weight required")
    if a.dtype != wt.dtype or a.ndim != 2 or a.shape[1] != wt.k:
        raise ValueError(f"Matching {wt.dtype} activation [M,{wt.k}] required")
    dev = nat.require_device(a, wt.tiles, bias)
    if a.stride(1) != 1 or (a.shape[0] > 1 and (a.stride(0) * 2) % 16) or a.data_ptr() % 16:
        a = a.contiguous()
    m = a.shape[0]
    out = torch.empty((m, wt.n), device=dev, dtype=a.dtype)
    lib = nat.library()
    need = lib.b2_w4a16_workspace_bytes(m, wt.n, wt.k, wt.group_size)
    if need and (workspace is None or workspace.numel() < need):
        # arrival counters at the end must start at zero; calls keep them zero
        workspace = torch.zeros(need, device=dev, dtype=torch.uint8)
    nat.check(lib.b2_w4a16_gemm(
        a.data_ptr(), nat.DTYPE_CODE[a.dtype], a.stride(0) if m > 1 else wt.k, wt.tiles.data_ptr(),
        wt.groups.data_ptr(), wt.group_size, m, wt.n, wt.k, nat.ptr(bias),
        nat.DTYPE_CODE[bias.dtype] if bias is not None else 0, out.data_ptr(), wt.n,
        None if not need else workspace.data_ptr(), need, nat.stream_ptr(dev)), "b2_w4a16_gemm")
    return out


def int4_linear_a16(a, p, *, bias=None, method="dequant", prepared=None, tile=(64, 64, 32),
                    num_warps=4, return_kernel=False):
    """16-bit activation x INT4 weight (reference int4_weight_gemm_v07.py:540-564).

    Methods "dequant" and "dot2" run the fused tcgen05 kernel (the dequantized
    weight never leaves shared memory); "prepared" uses a caller-owned
    `W4A16Weight`.  fp16 activations give fp16 output, bf16 give bf16.
    """
    if method not in ("dequant", "dot2", "prepared"):
        raise ValueError(method)
    if method == "prepared":
        if not isinstance(prepared, W4A16Weight):
            raise ValueError("W4A16Weight prepared weight required")
        if isinstance(p, PackedInt4):
            check_current(prepared, p)
        wt = prepared
    else:
        _validate(p)
        wt = None
    if a.dtype not in (torch.float16, torch.bfloat16) or a.ndim != 2:
        raise ValueError("Matching FP16/BF16 activation [M,K] required")
    k = wt.k if wt is not None else p.k
    n = wt.n if wt is not None else p.n
    if a.shape[1] != k or min(a.stride()) <= 0 or a.shape[0] * n >= 2**31:
        raise ValueError("Unsupported shape/stride")
    if bias is not None and (bias.dtype != a.dtype or bias.shape != (n,) or bias.device != a.device):
        raise ValueError("Bias [N] of the activation dtype required")
    nat.eager_only(a, bias)
    if method == "dot2" and (len(tile) != 3 or any(x not in (16, 32, 64, 128) for x in tile) or k % tile[2]):
        raise ValueError("Supported dot2 tile required")
    if wt is None:
        wt = prepare_w4a16(p, a.dtype)
    if wt.dtype != a.dtype:
        raise ValueError("Prepared weight dtype must match the activation dtype")
    out = w4a16_gemm(a, wt, bias)
    kernel = {"name": "w4a16_kernel (tcgen05 kind::f16, swap-AB)", "arch": "sm_100a"}
    return (out, kernel) if return_kernel else out


def dense_linear(a, w, bias=None):
    """16-bit dense GEMM on the tcgen05 kernel (kind::f16): a [M,K] @ w[N,K].T."""
    if a.dtype != w.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("fp16/bf16 operands of one dtype required")
    dev = nat.require_device(a, w, bias)
    m, k = a.shape
    n = w.shape[0]
    ones_m = torch.ones(m, device=dev, dtype=torch.float32)
    ones_n = torch.ones(1, device=dev, dtype=torch.float32)
    out = torch.empty((m, n), device=dev, dtype=a.dtype)
    kind = nat.KIND_BF16 if a.dtype == torch.bfloat16 else nat.KIND_F16
    return qgemm_raw(kind, a.view(torch.int16), w.view(torch.int16), ones_m, ones_n, bias,
                     nat.EPI_SEPARATE, out)


# ------------------------------------------------------------------ W4A8
_A8_METHODS = ("dot4", "dot4_words", "dot4_prepared", "dot4_split", "dot8")


def prepare_w4a8(p):
    """Caller-owned B200 W4A8 pack of a PackedInt4 (lossless: u = q + 8,
    zu = z + 8, fp32 scales kept)."""
    _validate(p)
    if p.k % 128:
        raise ValueError("W4A8 kernel needs K divisible by 128")
    lib = nat.library()
    tiles = torch.empty(lib.b2_w4a8_tiles_bytes(p.n, p.k), device=p.data.device, dtype=torch.uint8)
    groups = torch.empty(lib.b2_w4a8_groups_bytes(p.n, p.k, p.group_size), device=p.data.device,
                         dtype=torch.uint8)
    nat.check(lib.b2_w4a8_prepare(
        p.data.data_ptr(), int(p.layout == "kn"), int(p.order == "high"), p.scales.data_ptr(),
        p.zeros.data_ptr(), p.n, p.k, p.group_size, tiles.data_ptr(), groups.data_ptr(),
        nat.stream_ptr(p.data.device)), "b2_w4a8_prepare")
    return W4A8Weight(tiles, groups, p.n, p.k, p.group_size, source_stamp(p))


def int4_linear_a8(a, p, a_scale, *, bias=None, method="dot4", tile=(64, 64), num_warps=4,
                   prepared=None, integer=False, return_kernel=False):
    """Compute (A8 * row_scale) @ reconstructed W4.T, FP32 output
    (reference int4_weight_gemm_v07.py:476-537).

    Every method runs the tcgen05 kernel (csrc/w4a8.cu): per group an exact
    INT32 dot, times the fp32 group scale, accumulated in fp32 in group order,
    then times the row scale, plus bias -- bit-identical to the reference's
    grouped order.  `prepared` may be a W4A8Weight (this package's caller-owned
    pack); the reference's method-specific inputs (centered INT8 weight for
    dot4_prepared, the dot8 activation tuple) are validated like the
    reference and not needed.  integer=True returns the exact INT32 sum.
    """
    if isinstance(prepared, W4A8Weight):
        if isinstance(p, PackedInt4):
            check_current(prepared, p)
        wt = prepared
    else:
        _validate(p)
        wt = None
    n = wt.n if wt is not None else p.n
    k = wt.k if wt is not None else p.k
    nat.eager_only(a)
    if (a.ndim != 2 or a.dtype != torch.int8 or a.device.type != "cuda" or a.shape[1] != k
            or min(a.stride()) <= 0 or a.shape[0] * n >= 2**31):
        raise ValueError("Matching A8[M,K] required")
    m = a.shape[0]
    if (not integer and (a_scale is None or a_scale.shape not in ((m,), (m, 1)) or a_scale.device != a.device
                         or a_scale.dtype != torch.float32 or not a_scale.is_contiguous())):
        raise ValueError("Contiguous FP32 per-activation-row scale required")
    if bias is not None and (bias.shape != (n,) or bias.device != a.device or not bias.is_contiguous()
                             or not bias.is_floating_point()):
        raise ValueError("Floating bias [N] required")
    if len(tile) != 2 or any(x not in (8, 16, 32, 64, 128) for x in tile) or num_warps not in (4, 8):
        raise ValueError("Unsupported tile/warps")
    if k * 128 * 15 >= 2**31:
        raise ValueError("Integer accumulator bound exceeded")
    if method not in _A8_METHODS:
        raise ValueError(method)
    if method in ("dot4", "dot4_prepared", "dot4_split") and min(tile) < 16:
        raise ValueError("tl.dot tile dimensions must be >=16")
    if method == "dot4_prepared" and not isinstance(prepared, W4A8Weight):
        if (prepared is None or prepared.shape != (n, k) or prepared.dtype != torch.int8
                or prepared.device != a.device):
            raise ValueError("Centered INT8 prepared weight required")
    if method == "dot8" and prepared is not None and not isinstance(prepared, W4A8Weight):
        if not isinstance(prepared, tuple) or len(prepared) != 3:
            raise ValueError("Dot8 prepared tuple required")
    if wt is None:
        wt = prepare_w4a8(p)
    if a.stride(1) != 1 or a.stride(0) % 16 or a.data_ptr() % 16:
        a = a.contiguous()  # K % 128 == 0, so contiguous rows are 16-byte multiples
    dev = nat.require_device(a)
    out = torch.empty((m, n), device=dev, dtype=torch.int32 if integer else torch.float32)
    lib = nat.library()
    need = lib.b2_w4a8_workspace_bytes(m, k, wt.group_size)
    ws = torch.empty(max(need, 256), device=dev, dtype=torch.uint8)
    sa = a_scale.reshape(-1) if a_scale is not None else None
    nat.check(lib.b2_w4a8_gemm(
        a.data_ptr(), a.stride(0) if m > 1 else k, wt.tiles.data_ptr(), wt.groups.data_ptr(), wt.group_size,
        m, n, k, nat.ptr(sa), nat.ptr(bias), nat.DTYPE_CODE[bias.dtype] if bias is not None else 0,
        int(bool(integer)), out.data_ptr(), n, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
        "b2_w4a8_gemm")
    kernel = {"name": "w4a8_kernel (tcgen05 kind::i8, swap-AB, per-group TMEM drain)", "arch": "sm_100a"}
    return (out, kernel) if return_kernel else out
