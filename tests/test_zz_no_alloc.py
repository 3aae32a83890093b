"""The allocation-free entry point b2_quant_linear_noalloc, called through the
C ABI, must give the same bits as the workspace entry point b2_quant_linear.

It exists for callers that cannot hand the library a workspace (all device
memory owned by another allocator, plugin conventions that pass only inputs
and outputs, code that must not risk cudaMalloc's device-wide
synchronization); it stages the activation codes in a fixed device array
inside the library.  This file sorts last so that a run stopping at the first
failure has already run every other test; it also passes on its own.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import qlinear  # noqa: E402

EINVAL = 1


def _inputs(seed, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=g, device="cuda")
    x[:, torch.randperm(k, generator=g, device="cuda")[: max(1, k // 100)]] *= 20.0
    x = x.half()
    w = torch.randn((n, k), generator=g, device="cuda") * 0.02
    wq, sw = qlinear.quantize_weight(w, rotation_block=128)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.02).half()
    return x, wq, sw, bias


def _call(fn, x, wq, sw, bias, out, *extra):
    m, k = x.shape
    n = wq.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(nat.KIND_I8, x.data_ptr(), nat.F16, m, k, k, 128, wq.data_ptr(), k, n,
              sw.data_ptr(), n, bias.data_ptr(), nat.F16, nat.EPI_SEPARATE, out.data_ptr(),
              nat.F16, n, *extra, stream)


@pytest.mark.parametrize("m,n,k", [(1024, 3072, 3072), (4096, 12288, 3072), (37, 520, 256)])
def test_noalloc_matches_workspace_entry_point_twice(m, n, k):
    lib = nat.library()
    for seed in (1, 2):  # two calls in a row: the shared array keeps the last call's bytes
        x, wq, sw, bias = _inputs(seed * 1000 + m, m, n, k)
        ref = torch.empty((m, n), device="cuda", dtype=torch.float16)
        ws_bytes = lib.b2_quant_linear_workspace_bytes(m, k)
        ws = torch.empty(ws_bytes, device="cuda", dtype=torch.uint8)
        assert _call(lib.b2_quant_linear, x, wq, sw, bias, ref, ws.data_ptr(), ws_bytes) == 0
        got = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
        assert _call(lib.b2_quant_linear_noalloc, x, wq, sw, bias, got) == 0
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert nat.device_status() == 0


def test_noalloc_rejects_oversized_staging():
    lib = nat.library()
    cap = lib.b2_quant_linear_noalloc_max_bytes()
    k = 4096
    m = cap // k + 1  # staging of m x k codes no longer fits
    assert lib.b2_quant_linear_workspace_bytes(m, k) > cap
    x = torch.empty(1, device="cuda", dtype=torch.float16)  # never touched: rejected first
    status = lib.b2_quant_linear_noalloc(nat.KIND_I8, x.data_ptr(), nat.F16, m, k, k, 0,
                                         x.data_ptr(), k, 16, x.data_ptr(), 16, None, 0,
                                         nat.EPI_SEPARATE, x.data_ptr(), nat.F16, 16,
                                         torch.cuda.current_stream().cuda_stream)
    assert status == EINVAL
