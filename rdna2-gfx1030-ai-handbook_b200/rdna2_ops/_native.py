"""ctypes binding of librdna2_b200.so (the sm_100a C ABI in include/b2_qlinear.h).

Mirrors the reference's native-library loader (rdna2_ops/normalization.py:16-27):
one cached CDLL, explicit argtypes, launches on torch's current stream.
There is no fallback: every operator raises if the library or a B200-class
device is missing.
"""
from __future__ import annotations

import ctypes
import functools
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("RDNA2_B200_LIBRARY",
                               Path(__file__).with_name("lib") / "librdna2_b200.so"))

F32, F16, BF16, I32, E4M3, E5M2 = 0, 1, 2, 3, 4, 5
KIND_I8, KIND_E4M3, KIND_BF16, KIND_F16 = 0, 1, 2, 3
EPI_SEPARATE, EPI_FMA, EPI_KITCHEN, EPI_NONE = 0, 1, 2, 3

DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32,
              torch.float8_e4m3fn: E4M3, torch.float8_e5m2: E5M2}

_p, _i64, _int, _size = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t

# name -> (argtypes, restype); kept in step with include/b2_qlinear.h
SIGNATURES = {
    "b2_version": ([], _int),
    "b2_error_string": ([_int], ctypes.c_char_p),
    "b2_sm_count": ([], _int),
    "b2_set_gemm_path": ([_int], _int),
    "b2_set_prologue_path": ([_int], _int),
    "b2_set_w4a16_path": ([_int], _int),
    "b2_set_gather_store": ([_int], _int),
    "b2_pair_capacity": ([], _int),
    "b2_device_status": ([ctypes.POINTER(_int), _int], _int),
    "b2_act_quant": ([_p, _int, _i64, _i64, _i64, _int, _int, _p, _i64, _p, _p], _int),
    "b2_qgemm": ([_int, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _int, _int, _p,
                  _int, _i64, _p], _int),
    "b2_repack": ([_p, _int, _i64, _i64, _i64, _i64, _p, _i64, _p], _int),
    "b2_quant_linear_workspace_bytes": ([_i64, _i64], _size),
    "b2_quant_linear": ([_int, _p, _int, _i64, _i64, _i64, _int, _p, _i64, _i64, _p, _i64, _p,
                         _int, _int, _p, _int, _i64, _p, _size, _p], _int),
    "b2_w4a16_workspace_bytes": ([_i64, _i64, _i64, _int], _size),
    "b2_w4a16_gemm": ([_p, _int, _i64, _p, _p, _int, _i64, _i64, _i64, _p, _int, _p, _i64, _p, _size,
                       _p], _int),
    "b2_w4a16_tiles_bytes": ([_i64, _i64], _size),
    "b2_w4a8_tiles_bytes": ([_i64, _i64], _size),
    "b2_w4a8_groups_bytes": ([_i64, _i64, _int], _size),
    "b2_w4a8_workspace_bytes": ([_i64, _i64, _int], _size),
    "b2_w4a8_prepare": ([_p, _int, _int, _p, _p, _i64, _i64, _int, _p, _p, _p], _int),
    "b2_w4a8_gemm": ([_p, _i64, _p, _p, _int, _i64, _i64, _i64, _p, _p, _int, _int, _p, _i64, _p, _size, _p],
                     _int),
    "b2_w4a16_groups_bytes": ([_i64, _i64, _int], _size),
    "b2_w4a16_prepare": ([_p, _int, _int, _p, _p, _i64, _i64, _int, _int, _p, _p, _p], _int),
    "b2_fp8_decode": ([_p, _int, _i64, _i64, _i64, _int, _p, _i64, _p], _int),
    "b2_pack_int4": ([_p, _int, _i64, _i64, _i64, _int, _int, _int, _int, _p, _p, _p, _p, _p], _int),
    "b2_unpack_int4": ([_p, _int, _int, _p, _p, _i64, _i64, _int, _int, _p, _p], _int),
    "b2_ipc_handle_bytes": ([], _size),
    "b2_ipc_export": ([_p, _p, ctypes.POINTER(ctypes.c_uint64)], _int),
    "b2_ipc_import": ([_p, ctypes.c_uint64, ctypes.POINTER(_p)], _int),
    "b2_ipc_release": ([_p], _int),
    "b2_gather_state_bytes": ([], _size),
    "b2_quant_linear_gather": ([_int, _p, _int, _i64, _i64, _i64, _int, _p, _i64, _i64, _p, _i64, _p, _int,
                                _int, _int, _i64, _i64, _int, _int, ctypes.POINTER(_p), ctypes.POINTER(_p),
                                ctypes.c_uint32, _p, _size, _p], _int),
    "b2_gather_wait": ([_p, _int, ctypes.c_uint32, _p], _int),
    "b2_qgemm_gather": ([_int, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _int, _int, _int, _i64,
                         _i64, _int, _int, ctypes.POINTER(_p), ctypes.POINTER(_p), ctypes.c_uint32, _p], _int),
    "b2_peer_copy_2d": ([_p, _i64, _p, _i64, _i64, _i64, _p], _int),
    "b2_quant_linear_gather_ce": ([_int, _p, _int, _i64, _i64, _i64, _int, _p, _i64, _i64, _p, _i64, _p, _int,
                                   _int, _int, _i64, _i64, _int, _int, ctypes.POINTER(_p), ctypes.POINTER(_p),
                                   _int, _p, _size, _p], _int),
    "b2_gather_wait_ce": ([_p, _int, _int, _p], _int),
    "b2_shard_amax": ([_p, _int, _i64, _i64, _i64, _int, _int, _int, ctypes.POINTER(_p), ctypes.POINTER(_p),
                       ctypes.c_uint32, _p], _int),
    "b2_shard_exchange": ([_p, _int, _i64, _i64, _i64, _int, _int, _int, _int, ctypes.POINTER(_p), ctypes.POINTER(_p),
                           ctypes.c_uint32, ctypes.POINTER(_p), _i64, _i64, _p, ctypes.POINTER(_p), ctypes.c_uint32,
                           _p], _int),
    "b2_shard_codes": ([_p, _int, _i64, _i64, _i64, _int, _int, _int, _int, _p, ctypes.POINTER(_p), _i64, _i64,
                        _p, ctypes.POINTER(_p), ctypes.c_uint32, _p], _int),
    "b2_quant_linear_noalloc_max_bytes": ([], _size),
    "b2_quant_linear_noalloc": ([_int, _p, _int, _i64, _i64, _i64, _int, _p, _i64, _i64, _p, _i64,
                                 _p, _int, _int, _p, _int, _i64, _p], _int),
}


@functools.lru_cache(maxsize=1)
def library():
    if not LIB_PATH.is_file():
        raise RuntimeError(f"B200 kernel library missing at {LIB_PATH}; build it with "
                           "python rdna2-gfx1030-ai-handbook_b200/build.py")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


@functools.lru_cache(maxsize=16)
def _device_ok(index):
    major, minor = torch.cuda.get_device_capability(index)
    return major == 10


def require_device(*tensors):
    """All tensors on one CUDA device of compute capability 10.x (B200 class)."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("Inputs must be CUDA tensors on a B200 (sm_100) device")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("Inputs must share one CUDA device")
    if dev is None:
        raise ValueError("No CUDA tensor given")
    if not _device_ok(dev.index):
        raise ValueError("These kernels target sm_100 (B200); got compute capability "
                         + ".".join(map(str, torch.cuda.get_device_capability(dev.index))))
    return dev


def stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


def check(status, what):
    if status != 0:
        msg = library().b2_error_string(status)
        raise RuntimeError(f"{what} failed: {msg.decode() if msg else status}")


def ptr(t):
    return None if t is None else t.data_ptr()


def device_status(reset=False):
    """Synchronize and read the kernels' bounded-wait status word (0 = ok)."""
    torch.cuda.synchronize()
    v = _int(0)
    check(library().b2_device_status(ctypes.byref(v), int(bool(reset))), "b2_device_status")
    return v.value


def eager_only(*tensors):
    """Reference policy (rdna2_ops/int8_gemm.py:148-149, fp8_weight_gemm_v06.py:152-157):
    explicit eager inference only."""
    if (torch.compiler.is_compiling() or torch.cuda.is_current_stream_capturing()
            or torch.jit.is_tracing() or torch.jit.is_scripting()):
        raise RuntimeError("Only explicit eager calls are supported")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise ValueError("Autograd is unsupported")
