"""qwen_int8_gemm_candidate on the GPU (reference rdna2_ops/int8_gemm.py:274-330):
both bridge wrappers accelerated for fp32 inputs, every weight-scale branch
(per-row tensor, one-element tensor, Python number), with and without a bias,
bit-exact against the oracle's FMA epilogue (rounding="fused") applied to the
exact INT32 product of the bridge's own codes."""
import numpy as np
import pytest

import fake_qwen_bridge
import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops.int8_gemm import int8_gemm_dequant, qwen_int8_gemm_candidate  # noqa: E402


@pytest.fixture(autouse=True, scope="module")
def _status():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0


def _oracle(x, w, sb, bias, mode):
    codes, sa = fake_qwen_bridge.triton_quantize_rowwise(x.reshape(-1, x.shape[-1]))
    acc = oracle.gemm_s8(codes.cpu().numpy(), w.cpu().numpy())
    b = None if bias is None else bias.float().cpu().numpy()
    return oracle.epilogue_s32(acc, sa.cpu().numpy(), np.asarray(sb, np.float32), b, oracle.F32, mode,
                               oracle.F32)


@pytest.mark.parametrize("branch", ["per_row", "tensor_scalar", "python_scalar"])
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (37, 300, 1024), (300, 1000, 3072)])
def test_qwen_candidate_bit_exact(branch, with_bias, m, n, k):
    gen = torch.Generator(device="cuda").manual_seed(20261105 + m + n + k)
    x = torch.randn((2, m, k), generator=gen, device="cuda")
    w = torch.randint(-127, 128, (n, k), generator=gen, device="cuda", dtype=torch.int8)
    bias = (torch.randn(n, generator=gen, device="cuda") * 0.02) if with_bias else None
    per_row = torch.rand((n, 1), generator=gen, device="cuda") * 0.01 + 1e-4
    if branch == "per_row":
        fn, ws, sb = "triton_int8_linear_per_row", per_row, per_row.reshape(-1).cpu().numpy()
    elif branch == "tensor_scalar":
        fn, ws, sb = "triton_int8_linear", per_row[:1].clone(), per_row[:1].reshape(-1).cpu().numpy()
    else:
        fn, ws, sb = "triton_int8_linear", 0.0037, np.array([0.0037], np.float32)
    with qwen_int8_gemm_candidate(fake_qwen_bridge) as stats:
        y = getattr(fake_qwen_bridge, fn)(x, w, ws, bias=bias, compute_dtype=torch.float32)
    assert stats["hits"] == 1 and stats["fallbacks"] == 0
    assert y.shape == (2, m, n) and y.dtype == torch.float32
    ref = _oracle(x, w, sb, bias, oracle.EPI_FMA)
    assert np.array_equal(y.reshape(-1, n).cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_fused_and_separate_rounding_each_bit_exact():
    """rounding="fused" (one FMA) and "separate" (product and sum rounded
    apart) each match their oracle epilogue on the same operands; the two
    differ on some outputs, so the switch is live."""
    gen = torch.Generator(device="cuda").manual_seed(20261106)
    m, n, k = 200, 640, 2048
    a = torch.randint(-127, 128, (m, k), generator=gen, device="cuda", dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=gen, device="cuda", dtype=torch.int8)
    sa = torch.rand(m, generator=gen, device="cuda") * 0.01 + 1e-4
    sb = torch.rand(n, generator=gen, device="cuda") * 0.01 + 1e-4
    bias = torch.randn(n, generator=gen, device="cuda")
    acc = oracle.gemm_s8(a.cpu().numpy(), w.cpu().numpy())
    outs = {}
    for rounding, mode in (("fused", oracle.EPI_FMA), ("separate", oracle.EPI_SEPARATE)):
        y = int8_gemm_dequant(a, w.T, sa, sb, bias, rounding=rounding)
        ref = oracle.epilogue_s32(acc, sa.cpu().numpy(), sb.cpu().numpy(), bias.cpu().numpy(), oracle.F32,
                                  mode, oracle.F32)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), rounding
        outs[rounding] = y
    assert not torch.equal(outs["fused"], outs["separate"])
