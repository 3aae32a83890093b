"""The production boundary on the GPU: Kitchen's eager int8_linear export,
replaced by the B200 backend, against the reference backend's own output
(golden, produced by running production/MOSS_RDNA2_INT8/backend.py) and the
oracle's Kitchen epilogue for fp16/bf16 and ConvRot calls."""
import numpy as np
import pytest

import fake_kitchen
import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops.int8_gemm import int8_matmul, moss_int8_gemm_candidate  # noqa: E402

ODT = {torch.float32: oracle.F32, torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}


def bits(t):
    t = t.detach().cpu()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


@pytest.fixture()
def installed():
    k = fake_kitchen.install()
    import MOSS_RDNA2_INT8.backend as be
    k.quant._int8_matmul_accumulate = int8_matmul
    be.install_backend(int8_matmul)
    yield k
    be.disable_backend()
    k.uninstall()


@pytest.mark.parametrize("case", [0, 1, 2])
def test_kitchen_dispatch_matches_reference_backend(golden, installed, case):
    g = golden("moss_backend_fp32.npz")
    bias = g[f"c{case}_bias"] if f"c{case}_bias" in g.files else None
    fn = installed.registry.get_implementation("int8_linear", backend="eager")
    y = fn(torch.from_numpy(g[f"c{case}_x"]).cuda(), torch.from_numpy(g[f"c{case}_w"]).cuda(),
           torch.from_numpy(g[f"c{case}_ws"]).cuda(),
           None if bias is None else torch.from_numpy(bias).cuda(), out_dtype=torch.float32)
    assert np.array_equal(bits(y).view(np.uint32), g[f"c{case}_y"].view(np.uint32))


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("convrot", [False, True])
def test_kitchen_epilogue_all_dtypes(installed, x_dtype, out_dtype, convrot):
    rng = np.random.default_rng(7)
    m, n, k = 3 * 65, 400, 512
    x = rng.standard_normal((2, m // 2 + 1, k)).astype(np.float32)   # 3-D input, leading dims kept
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, 256 if convrot else 0))
    bias = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float32)).to(torch.bfloat16)
    xt = torch.from_numpy(x).to(x_dtype).cuda()
    fn = installed.registry.get_implementation("int8_linear", backend="eager")
    y = fn(xt, torch.from_numpy(wq).cuda(), torch.from_numpy(sw).cuda(), bias.cuda(),
           out_dtype=out_dtype, convrot=convrot, convrot_groupsize=256)
    assert y.shape == (2, m // 2 + 1, n) and y.dtype == out_dtype
    ref = oracle.w8a8_linear(bits(xt).reshape(-1, k), ODT[x_dtype], 256 if convrot else 0, wq, sw,
                             bits(bias), oracle.BF16, oracle.EPI_KITCHEN, ODT[out_dtype])
    got = bits(y).reshape(-1, n)
    assert np.array_equal(got.view(np.uint32) if got.dtype == np.float32 else got,
                          ref.view(np.uint32) if ref.dtype == np.float32 else ref)


def test_input_act_and_residual_use_kitchen_helpers(installed):
    x = torch.randn(4, 64, device="cuda")
    w = torch.randint(-127, 128, (32, 64), dtype=torch.int8, device="cuda")
    ws = torch.full((32,), 0.01, device="cuda")
    res = torch.randn(4, 32, device="cuda")
    fn = installed.registry.get_implementation("int8_linear", backend="eager")
    base = fn(x * 2, w, ws, out_dtype=torch.float32)
    y = fn(x, w, ws, out_dtype=torch.float32, input_act="situ", residual=res)
    assert installed.calls["input_act"] == 1 and installed.calls["residual"] == 1
    assert torch.equal(y, base + res)


def test_moss_candidate_context(installed):
    """moss_int8_gemm_candidate: fused prologue + GEMM with the separate fp32
    epilogue (reference int8_gemm.py:231-263), accelerated for fp16 too."""
    rng = np.random.default_rng(8)
    x = rng.standard_normal((70, 384)).astype(np.float32)
    w = (rng.standard_normal((256, 384)) * 0.02).astype(np.float32)
    wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, 128))
    bias = (rng.standard_normal(256) * 0.02).astype(np.float32)
    with moss_int8_gemm_candidate(tile=(64, 128, 64), num_warps=4, num_stages=2, group_m=8) as stats:
        y = installed.eager.int8_linear(torch.from_numpy(x).cuda(), torch.from_numpy(wq).cuda(),
                                        torch.from_numpy(sw).cuda(), torch.from_numpy(bias).cuda(),
                                        out_dtype=torch.float32, convrot=True, convrot_groupsize=128)
    assert stats["hits"] == 1
    ref = oracle.w8a8_linear(x, oracle.F32, 128, wq, sw, bias, oracle.F32, oracle.EPI_SEPARATE, oracle.F32)
    assert np.array_equal(bits(y).view(np.uint32), ref.view(np.uint32))
    assert nat.device_status() == 0
