"""The float-output contract on the CPU: the reference's own PyTorch math
(F.linear on the dequantized 16-bit weight, int4_weight_gemm_v07.py:540-564
method "dequant"; fp8_weight_gemm_v06.py:166-167 "upcast") is measured
against the f64 value of the same math with the rule the GPU tests use
(conftest.assert_within_ulp): 1 ulp of the output type plus 2^-20 * sum|a*w|.
A bare 1-ulp rule is not met by any fp32 accumulation on outputs that cancel
(|y| << sum|a*w|); the test records how many outputs the reference math
itself leaves outside a bare ulp, and holds it to the same rule."""
import numpy as np
import pytest

import oracle
from conftest import assert_within_ulp, ulp_of

torch = pytest.importorskip("torch")

from rdna2_ops import int4_weight_gemm_v07 as i4  # noqa: E402

KIND = {torch.bfloat16: ("bf16", oracle.BF16), torch.float16: ("fp16", oracle.F16)}


def test_ulp_of():
    assert ulp_of(1.0, "bf16") == 2.0 ** -7 and ulp_of(1.5, "fp16") == 2.0 ** -10
    assert ulp_of(0.0, "fp16") == 2.0 ** -24 and ulp_of(-3.0, "fp32") == 2.0 ** -22


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_reference_torch_math_meets_the_same_rule(dtype):
    kind, code = KIND[dtype]
    gen = torch.Generator().manual_seed(20261107)
    m, n, k = 32, 2048, 4096
    w = torch.randn((n, k), generator=gen) * 0.02
    p = i4.pack_int4_cpu(w, group_size=128, symmetric=False)
    s16 = p.scales.to(dtype).float().numpy()
    w32 = oracle.dequant_int4(p.data.numpy(), s16, p.zeros.float().numpy(), 128, out_dtype=code)
    w16 = torch.from_numpy(w32).to(dtype)                   # exact: values already rounded to dtype
    a = torch.randn((m, k), generator=gen).to(dtype)
    y = torch.nn.functional.linear(a, w16)                  # the reference's PyTorch math
    a64, w64 = a.double().numpy(), w16.double().numpy()
    ref, absref = a64 @ w64.T, np.abs(a64) @ np.abs(w64).T
    got = y.double().numpy()
    bare = int((np.abs(got - ref) > ulp_of(got, kind)).sum())
    print(f"reference torch math, {kind}: {bare} of {got.size} outputs outside a bare ulp")
    assert_within_ulp(got, ref, absref, kind, f"torch F.linear {kind}")
