"""ConvRot INT8 checkpoints on disk, and caller-owned weight packs.

On-disk format: the ConvRot INT8 safetensors files the reference benchmarks
read (MOSS `moss_image_sft_int8_convrot.safetensors`, Qwen
`qwen_image_2.1_int8_convrot.safetensors`; rdna2-ops/bench_int4_v07.py:39-43,
193-200).  Each quantized linear `<name>` is stored as

  `<name>.weight`        int8 [N, K], row-major -- the layout the production
                         `int8_linear` reads through a `weight.T` view
                         (production/MOSS_RDNA2_INT8/backend.py:100-124)
  `<name>.weight_scale`  fp32 [N] per output channel, or a scalar
  `<name>.bias`          optional, [N]

with the block-Hadamard (ConvRot) rotation already folded into the weight, so
activations are rotated at run time with the same block.  Other tensors of
a file are passed through untouched.

B200 note on "pre-transposed" packs: on gfx1030 a pre-transposed contiguous
RHS ran the GEMM 2.16-2.55x faster than the `weight.T` view
(production/README.md:83-101), but the reference left it out because a
pointer-keyed cache cannot follow weight lifetimes (offload, LoRA,
requantization).  The tcgen05 GEMM here reads the stored [N, K] weight as its
K-major operand directly (TMA, no copy), so the view path already is the fast
path and no INT8 pack exists to go stale.  The INT4 formats do need a
one-time conversion (`prepare_w4a16`, `prepare_w4a8`); those packs are
caller-owned, carry a stamp of the PackedInt4 they came from, and are
rejected once that source changes (`check_current`), instead of being
looked up by address.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass
from pathlib import Path

import torch

_SCALE_SUFFIX = ".weight_scale"


@dataclass
class Int8Linear:
    """One ConvRot INT8 linear: weight int8 [N, K], weight_scale fp32 [N] or
    [1], optional bias [N]."""
    weight: torch.Tensor
    weight_scale: torch.Tensor
    bias: torch.Tensor | None = None

    def __post_init__(self):
        validate_int8_linear(self.weight, self.weight_scale, self.bias)

    @property
    def out_features(self):
        return self.weight.shape[0]

    @property
    def in_features(self):
        return self.weight.shape[1]

    def to(self, device):
        b = None if self.bias is None else self.bias.to(device)
        return Int8Linear(self.weight.to(device), self.weight_scale.to(device), b)

    def __call__(self, x, *, rotation_block=128, out_dtype=None, epilogue="separate"):
        """The fused linear: rotate x by `rotation_block` (None for a weight
        quantized without rotation), quantize per token, GEMM, epilogue."""
        from .qlinear import w8a8_linear
        return w8a8_linear(x, self.weight, self.weight_scale.reshape(-1), self.bias,
                           rotation_block=rotation_block, out_dtype=out_dtype, epilogue=epilogue)


def validate_int8_linear(weight, weight_scale, bias=None):
    """The checks of the production backend (backend.py:100-110): int8 [N, K]
    weight, fp32-convertible scale with 1 or N entries, bias [N]."""
    if not isinstance(weight, torch.Tensor) or weight.dtype != torch.int8 or weight.ndim != 2:
        raise TypeError("ConvRot INT8 weight must be an int8 [N,K] tensor")
    if not isinstance(weight_scale, torch.Tensor) or not weight_scale.is_floating_point():
        raise TypeError("weight_scale must be a floating-point tensor")
    if weight_scale.numel() not in (1, weight.shape[0]):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got "
                         f"{tuple(weight_scale.shape)} for weight shape {tuple(weight.shape)}")
    if bias is not None and (not isinstance(bias, torch.Tensor) or bias.numel() != weight.shape[0]):
        raise ValueError("bias must hold one value per output channel")


def digest(t):
    """SHA-256 of a tensor's bytes (the provenance hash the reference records
    per weight, bench_int4_v07.py:46-47)."""
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def read_weight(path, name, *, device="cpu"):
    """(weight, scale, metadata) of `name` (a `*.weight` key), as the
    reference's `read_weight` (bench_int4_v07.py:193-200) reads it; scale is
    None when the file has no `*.weight_scale` for it."""
    from safetensors import safe_open
    path = Path(path)
    if not name.endswith(".weight"):
        raise ValueError("name must be a '*.weight' key")
    with safe_open(str(path), framework="pt", device=str(device)) as f:
        keys = set(f.keys())
        if name not in keys:
            raise KeyError(name)
        w = f.get_tensor(name)
        sname = name[: -len(".weight")] + _SCALE_SUFFIX
        scale = f.get_tensor(sname).reshape(-1) if sname in keys else None
    md = {"file": str(path), "name": name, "dtype": str(w.dtype), "shape": list(w.shape),
          "tensor_sha256": digest(w), "scale_sha256": None if scale is None else digest(scale)}
    return w, scale, md


def load_int8_linears(path, *, device="cuda", names=None):
    """Every ConvRot INT8 linear of a safetensors file: {name: Int8Linear} for
    each int8 `<name>.weight` with a `<name>.weight_scale` (and its
    `<name>.bias` when present), loaded onto `device`.  `names` restricts the
    result to those linears (KeyError when one is missing)."""
    from safetensors import safe_open
    out = {}
    with safe_open(str(path), framework="pt", device=str(device)) as f:
        keys = set(f.keys())
        found = sorted(k[: -len(_SCALE_SUFFIX)] for k in keys if k.endswith(_SCALE_SUFFIX)
                       and k[: -len(_SCALE_SUFFIX)] + ".weight" in keys)
        if names is not None:
            missing = [n for n in names if n not in found]
            if missing:
                raise KeyError(f"no ConvRot INT8 linear named {missing[0]!r} in {path}")
            found = list(names)
        for name in found:
            w = f.get_tensor(name + ".weight")
            if w.dtype != torch.int8:
                continue  # a scaled non-INT8 weight: not this format
            s = f.get_tensor(name + _SCALE_SUFFIX).float().reshape(-1)
            b = f.get_tensor(name + ".bias") if name + ".bias" in keys else None
            out[name] = Int8Linear(w, s, b)
    return out


def save_int8_linears(path, linears, *, extra=None, metadata=None):
    """Write {name: Int8Linear} (plus pass-through tensors `extra`) in the
    ConvRot INT8 safetensors layout."""
    from safetensors.torch import save_file
    tensors = {}
    for name, lin in linears.items():
        if not isinstance(lin, Int8Linear):
            lin = Int8Linear(*lin)
        tensors[name + ".weight"] = lin.weight.detach().contiguous().cpu()
        tensors[name + _SCALE_SUFFIX] = lin.weight_scale.detach().float().contiguous().cpu()
        if lin.bias is not None:
            tensors[name + ".bias"] = lin.bias.detach().contiguous().cpu()
    for k, v in (extra or {}).items():
        if k in tensors:
            raise ValueError(f"duplicate key {k!r}")
        tensors[k] = v.detach().contiguous().cpu()
    save_file(tensors, str(path), metadata=metadata)


def quantize_convrot(w, bias=None, *, rotation_block=128):
    """Float [N, K] weight -> Int8Linear with the block-Hadamard rotation
    folded in (per-output-channel absmax / 127, ties to even) on the GPU."""
    from .qlinear import quantize_weight
    wq, sw = quantize_weight(w, rotation_block=rotation_block)
    return Int8Linear(wq, sw, bias)


# ------------------------------------------------- INT4 pack invalidation
def source_stamp(p):
    """Identity of a PackedInt4's tensors: storage address, shape and the
    in-place version counter of data, scales and zeros.  Any in-place update
    (a LoRA merge, a requantization) or a replaced tensor changes it."""
    return tuple((t.data_ptr(), tuple(t.shape), t._version) for t in (p.data, p.scales, p.zeros))


def check_current(prepared, p):
    """Raise when `prepared` (a W4A16Weight / W4A8Weight carrying a source
    stamp) was not made from the current state of PackedInt4 `p`."""
    stamp = getattr(prepared, "source", None)
    if stamp is not None and p is not None and stamp != source_stamp(p):
        raise ValueError("Prepared INT4 weight is stale: its PackedInt4 changed since it was prepared "
                         "(prepare it again after weight or LoRA updates)")
