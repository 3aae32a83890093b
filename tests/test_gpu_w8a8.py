"""GPU parity of the W8A8 / FP8 hot path against the CPU oracle and the
reference's golden vectors.  Integer work (codes, INT32 accumulators) is
bit-exact; fp32/fp16/bf16 outputs of the INT8 path are bit-exact too (the
epilogue reproduces the reference rounding order).  FP8 outputs: within the
1 bf16 ulp plus the fp32 accumulation term (conftest.assert_within_ulp)."""
import numpy as np
import pytest

import oracle
from conftest import assert_within_ulp, outlier_activations

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rdna2_ops  # noqa: E402
from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import qlinear  # noqa: E402

ODT = {torch.float32: oracle.F32, torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}
EPI = {"separate": oracle.EPI_SEPARATE, "fused": oracle.EPI_FMA, "kitchen": oracle.EPI_KITCHEN}


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(t):
    """Tensor -> numpy storage bits matching the oracle conventions."""
    t = t.detach().cpu()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def same_bits(t, ref):
    got = bits(t)
    if got.dtype == np.float32:
        return np.array_equal(got.view(np.uint32), np.asarray(ref, np.float32).view(np.uint32))
    return np.array_equal(got, ref)


def x_tensor(x32, dtype):
    return torch.from_numpy(x32).to(dtype).cuda()


def x_bits(xt):
    return bits(xt)


@pytest.fixture(params=["single256", "single128", "pair256", "pair192", "pair256s", "pair192s", "splitk"])
def gemm_path(request):
    qlinear.set_gemm_path(request.param)
    yield request.param
    qlinear.set_gemm_path("auto")


@pytest.fixture(autouse=True, scope="module")
def _device_status_clean():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0, "a kernel's bounded wait gave up"


# ------------------------------------------------------- golden: INT8 GEMM
@pytest.mark.parametrize("key", ["weight_nk_vector", "weight_nk_scalar", "rhs_kn_vector",
                                 "rhs_kn_scalar"])
def test_int8_known_answer(golden, key, gemm_path):
    """bench_int8_gemm.py:181-203 on the GPU: offset+padded A view, weight.T view
    and contiguous [K,N] B, INT32 exact, FP32 dequant bitwise."""
    g = golden("int8_known_answer.npz")
    a = cuda(g[key + "_a_store"])[1:38, 1:80]
    w = cuda(g[key + "_w"])
    b = w.T if key.startswith("weight_nk") else w.T.contiguous()
    acc = rdna2_ops.int8_matmul(a, b)
    assert acc.dtype == torch.int32 and np.array_equal(acc.cpu().numpy(), g[key + "_acc"])
    out = rdna2_ops.int8_gemm_dequant(a, b, cuda(g[key + "_sa"]), cuda(g[key + "_sb"]),
                                      cuda(g[key + "_bias"]))
    assert same_bits(out, g[key + "_ref"])


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (1, 16, 16), (37, 53, 79), (129, 257, 33),
                                   (128, 256, 128), (300, 200, 1000), (513, 640, 3072), (1024, 9472, 384),
                                   (64, 96, 131071 // 8), (16, 5120, 640), (32, 300, 4096), (5, 20000, 256)])
def test_int8_matmul_exact(m, n, k, gemm_path):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    w = rng.integers(-128, 128, (n, k), dtype=np.int8)
    ref = oracle.gemm_s8(a, w)
    got = rdna2_ops.int8_matmul(cuda(a), cuda(w).T)
    assert np.array_equal(got.cpu().numpy(), ref)
    got2 = rdna2_ops.int8_matmul(cuda(a), cuda(w).T.contiguous())      # [K,N] layout
    assert np.array_equal(got2.cpu().numpy(), ref)


def test_int8_accumulator_extremes(gemm_path):
    k = 4096
    a = np.full((130, k), -128, np.int8)
    w = np.full((140, k), -128, np.int8)
    w[1::2] = 127
    got = rdna2_ops.int8_matmul(cuda(a), cuda(w).T).cpu().numpy()
    assert np.array_equal(got, oracle.gemm_s8(a, w))


@pytest.mark.parametrize("rounding", ["separate", "fused"])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("scalar", [False, True])
def test_int8_gemm_dequant_epilogues(rounding, out_dtype, scalar, gemm_path):
    rng = np.random.default_rng(11)
    m, n, k = 200, 264, 512
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    w = rng.integers(-127, 128, (n, k), dtype=np.int8)
    sa = (rng.random(m) * 0.02 + 0.001).astype(np.float32)
    sb = (rng.random(1 if scalar else n) * 0.02 + 0.001).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    acc = oracle.gemm_s8(a, w)
    ref = oracle.epilogue_s32(acc, sa, sb, bias, oracle.F32, EPI[rounding], ODT[out_dtype])
    out = rdna2_ops.int8_gemm_dequant(cuda(a), cuda(w).T, cuda(sa), cuda(sb), cuda(bias),
                                      rounding=rounding, out_dtype=out_dtype)
    assert same_bits(out, ref)


@pytest.mark.parametrize("m,n,k", [(1, 5120, 5120), (13, 1000, 640), (32, 4096, 1024), (3, 20000, 256)])
@pytest.mark.parametrize("rounding", ["separate", "fused", "kitchen"])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_int8_decode_split_k_epilogues(m, n, k, rounding, out_dtype):
    """M <= 32 runs the split-K cluster kernel (automatic choice): partial
    int32 sums from every CTA of a cluster, reduced in the leader, then the
    same epilogue rounding as every other path."""
    rng = np.random.default_rng(m * 31 + n + k)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    w = rng.integers(-127, 128, (n, k), dtype=np.int8)
    sa = (rng.random(m) * 0.02 + 0.001).astype(np.float32)
    sb = (rng.random(n) * 0.02 + 0.001).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    acc = oracle.gemm_s8(a, w)
    assert np.array_equal(rdna2_ops.int8_matmul(cuda(a), cuda(w).T).cpu().numpy(), acc)
    ref = oracle.epilogue_s32(acc, sa, sb, bias, oracle.F32, EPI[rounding], ODT[out_dtype])
    if rounding == "kitchen":
        out = torch.empty((m, n), device="cuda", dtype=out_dtype)
        qlinear.qgemm_raw(nat.KIND_I8, cuda(a), cuda(w), cuda(sa), cuda(sb), cuda(bias), nat.EPI_KITCHEN, out)
    else:
        out = rdna2_ops.int8_gemm_dequant(cuda(a), cuda(w).T, cuda(sa), cuda(sb), cuda(bias), rounding=rounding,
                                          out_dtype=out_dtype)
    assert same_bits(out, ref)


@pytest.mark.parametrize("m", [3, 300])
def test_back_to_back_launches_without_sync(m):
    """The fused linear's GEMM is launched with programmatic serialization
    and may start while its prologue runs.  Weights quantized by the
    previous kernel, and a chain of linears each reading the previous one's
    output, must give the same bits as the same calls synchronised one by
    one."""
    rng = np.random.default_rng(m)
    k, n = 1024, 2048
    w1 = torch.from_numpy((rng.standard_normal((n, k)) * 0.03).astype(np.float32)).cuda()
    w2 = torch.from_numpy((rng.standard_normal((k, n)) * 0.03).astype(np.float32)).cuda()
    x = torch.from_numpy(outlier_activations(rng, m, k)).cuda().half()

    def chain(sync):
        wq1, sw1 = qlinear.quantize_weight(w1, rotation_block=128)
        if sync:
            torch.cuda.synchronize()
        y1 = rdna2_ops.w8a8_linear(x, wq1, sw1, None, rotation_block=128, out_dtype=torch.float16)
        if sync:
            torch.cuda.synchronize()
        wq2, sw2 = qlinear.quantize_weight(w2, rotation_block=128)
        if sync:
            torch.cuda.synchronize()
        y2 = rdna2_ops.w8a8_linear(y1, wq2, sw2, None, rotation_block=128, out_dtype=torch.float16)
        # a GEMM whose weight operand the kernel just before it writes
        qx, sx = rdna2_ops.act_quant(x, rotation_block=128)
        wq3, sw3 = qlinear.quantize_weight(w1, rotation_block=128)
        if sync:
            torch.cuda.synchronize()
        y3 = rdna2_ops.int8_gemm_dequant(qx, wq3.T, sx, sw3, None)
        torch.cuda.synchronize()
        return y1.clone(), y2.clone(), y3.clone()

    ref = chain(True)
    for _ in range(3):
        got = chain(False)
        for g, r in zip(got, ref):
            assert same_bits(g, bits(r))


# ----------------------------------------------------- prologue (act_quant)
@pytest.fixture(params=["shuffle", "lane"])
def prologue_path(request):
    qlinear.set_prologue_path(request.param)
    yield request.param
    qlinear.set_prologue_path("auto")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k,block", [(3072, 128), (3072, None), (3072, 256), (3072, 1024),
                                     (384, 128), (4096, 128), (5120, 128), (12288, 128),
                                     (8192, 2048), (16384, 256), (80, 16), (24, None)])
def test_act_quant_bit_exact(dtype, k, block, prologue_path):
    rng = np.random.default_rng(k + (block or 0))
    m = 67
    x32 = outlier_activations(rng, m, k)
    x32[3] = 0.0                                   # all-zero row -> scale 1, codes 0
    xt = x_tensor(x32, dtype)
    q, s = rdna2_ops.act_quant(xt, rotation_block=block)
    ref_q, ref_s = oracle.act_quant_int8(x_bits(xt), ODT[dtype], block or 0)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), ref_q)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_act_quant_exact_ties_round_to_even(dtype, prologue_path):
    """Rows whose scale is exactly 1 (absmax 127) with values on x.5: both
    kernels' quantizers (the shuffle kernel's fast path with its exact
    fallback, the lane kernel's FMA-corrected quotient) must round ties to
    even, like the oracle."""
    k = 1024
    x32 = np.zeros((4, k), dtype=np.float32)
    ties = np.array([0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5, 126.5, -126.5, 64.5], dtype=np.float32)
    for r in range(4):
        x32[r, 0] = 127.0
        x32[r, 1:1 + ties.size] = ties * (1 if r % 2 == 0 else -1)
    xt = x_tensor(x32, dtype)
    q, s = rdna2_ops.act_quant(xt, rotation_block=None)
    ref_q, ref_s = oracle.act_quant_int8(x_bits(xt), ODT[dtype], 0)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert list(q.cpu().numpy()[0, 1:5]) == [0, 2, 2, 4]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("block", [None, 128])
def test_act_quant_extreme_scales(dtype, block, prologue_path):
    """Row scales far from 1: below 2^-60 and above 2^60 (the lane kernel's
    exact power-of-two rescaling), subnormal (clamped IEEE division), and
    rows of exact ties at scale 1, against the oracle's IEEE division."""
    rng = np.random.default_rng(11)
    x32 = outlier_activations(rng, 9, 3072)
    x32[0] *= 1e-25
    x32[1] *= 1e-39
    x32[2] *= 1e30
    x32[3] *= 7e-20
    x32[4] *= 3e19
    x32[5] *= 1e-44 if dtype == torch.float32 else 1e-40
    x32[6] = np.round(x32[6] * 2.0) / 2.0
    xt = x_tensor(x32, dtype)
    q, s = rdna2_ops.act_quant(xt, rotation_block=block)
    ref_q, ref_s = oracle.act_quant_int8(x_bits(xt), ODT[dtype], block or 0)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), ref_q)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k,block", [(5120, None), (3072, 128), (4096, 1024), (384, 128), (80, 16)])
def test_act_quant_e4m3_bit_exact(dtype, k, block, prologue_path):
    """Per-token e4m3 codes (scale absmax/448, e4m3_rn_sat(RN(v/s))) on both
    prologue kernels, with and without rotation, against the oracle."""
    rng = np.random.default_rng(5 + k)
    x32 = outlier_activations(rng, 33, k)
    x32[2] = 0.0
    xt = x_tensor(x32, dtype)
    q, s = rdna2_ops.act_quant(xt, rotation_block=block, quant="e4m3")
    ref_q, ref_s = oracle.quant_rows_e4m3(oracle.rotate_rows(x_bits(xt), ODT[dtype], block or 0))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), ref_q)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_act_quant_e4m3_extreme_scales_and_grid_ties(dtype, prologue_path):
    """e4m3 codes for scales below 2^-60, above 2^60 and subnormal, and for
    rows whose quotients fall exactly between two e4m3 values (scale 1:
    absmax 448) or at the saturation edge."""
    rng = np.random.default_rng(12)
    x32 = outlier_activations(rng, 8, 3072)
    x32[0] *= 1e-25
    x32[1] *= 1e-39
    x32[2] *= 1e30
    x32[3] *= 1e-44 if dtype == torch.float32 else 1e-40
    x32[4] = 0.0
    x32[4, 0] = 448.0
    grid_ties = np.array([1.0625, 1.1875, 17.0, 19.0, 240.0, 272.0, 432.0, 440.0, 0.0068359375], np.float32)
    x32[4, 1:1 + grid_ties.size] = grid_ties
    x32[5] = -x32[4]
    xt = x_tensor(x32, dtype)
    q, s = rdna2_ops.act_quant(xt, quant="e4m3")
    ref_q, ref_s = oracle.quant_rows_e4m3(oracle.rotate_rows(x_bits(xt), ODT[dtype], 0))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), ref_q)


def test_act_quant_strided_rows():
    rng = np.random.default_rng(6)
    big = outlier_activations(rng, 40, 1000)
    xt = x_tensor(big, torch.float16)[:, 8:8 + 768]   # row stride 1000, offset 8
    q, s = rdna2_ops.act_quant(xt, rotation_block=256)
    ref_q, ref_s = oracle.act_quant_int8(x_bits(xt), oracle.F16, 256)
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(s.cpu().numpy(), ref_s)


# ------------------------------------------------------ fused W8A8 linear
def _weights(rng, n, k, block):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, block or 0))
    return w, wq, sw


@pytest.mark.parametrize("m,n,k,block", [(1, 64, 128, 128), (37, 53, 96, None),
                                         (128, 256, 3072, 128), (200, 384, 512, 256),
                                         (333, 4000, 1024, 128)])
@pytest.mark.parametrize("epilogue", ["separate", "kitchen", "fused"])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_w8a8_linear_bit_exact(m, n, k, block, epilogue, out_dtype, gemm_path):
    rng = np.random.default_rng(m + n + k)
    x32 = outlier_activations(rng, m, k)
    _, wq, sw = _weights(rng, n, k, block)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    xt = x_tensor(x32, torch.float16)
    bias_t = torch.from_numpy(bias).to(torch.float16).cuda()
    y = rdna2_ops.w8a8_linear(xt, cuda(wq), cuda(sw), bias_t, rotation_block=block,
                              out_dtype=out_dtype, epilogue=epilogue)
    ref = oracle.w8a8_linear(x_bits(xt), oracle.F16, block or 0, wq, sw, bits(bias_t),
                             oracle.F16, EPI[epilogue], ODT[out_dtype])
    assert same_bits(y, ref)


def test_quantize_weight_folds_rotation_bit_exact():
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((300, 3072)) * 0.02).astype(np.float32)
    q, s = qlinear.quantize_weight(cuda(w), rotation_block=128)
    rq, rs = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, 128))
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_config1_full_size_bit_exact():
    """X fp16 [1024,3072] with 1% outlier channels, W int8
    [3072,3072] per-channel, fp16 bias, fp16 out, no rotation."""
    rng = np.random.default_rng(20261106)
    m, n, k = 1024, 3072, 3072
    x32 = outlier_activations(rng, m, k)
    _, wq, sw = _weights(rng, n, k, None)
    bias_t = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float32)).half().cuda()
    xt = x_tensor(x32, torch.float16)
    y = rdna2_ops.w8a8_linear(xt, cuda(wq), cuda(sw), bias_t, out_dtype=torch.float16)
    ref = oracle.w8a8_linear(x_bits(xt), oracle.F16, 0, wq, sw, bits(bias_t), oracle.F16,
                             oracle.EPI_SEPARATE, oracle.F16)
    assert same_bits(y, ref)


def test_config2_full_size_bit_exact_and_deterministic():
    """BASELINE config 2 at full size (4096 x 12288 x 3072, rotation 128):
    codes and scales bit-exact for every row, all 50.3 M fp16 outputs
    bit-exact against the oracle's exact INT32 GEMM and epilogue, two runs
    bitwise identical."""
    rng = np.random.default_rng(20261105)
    m, n, k = 4096, 12288, 3072
    xt = x_tensor(outlier_activations(rng, m, k), torch.float16)
    wt = torch.from_numpy((rng.standard_normal((n, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(wt, rotation_block=128)
    bias_t = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float32)).half().cuda()
    y1 = rdna2_ops.w8a8_linear(xt, wq, sw, bias_t, rotation_block=128, out_dtype=torch.float16)
    y2 = rdna2_ops.w8a8_linear(xt, wq, sw, bias_t, rotation_block=128, out_dtype=torch.float16)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    q, s = rdna2_ops.act_quant(xt, rotation_block=128)
    rq, rs = oracle.act_quant_int8(bits(xt), oracle.F16, 128)
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    rwq, rsw = oracle.quant_rows_int8(oracle.rotate_rows(wt.cpu().numpy(), oracle.F32, 128))
    assert np.array_equal(wq.cpu().numpy(), rwq) and np.array_equal(sw.cpu().numpy(), rsw)
    acc = oracle.gemm_s8(rq, rwq)
    ref = oracle.epilogue_s32(acc, rs, rsw, bits(bias_t), oracle.F16, oracle.EPI_SEPARATE, oracle.F16)
    assert np.array_equal(bits(y1), ref)


# -------------------------------------------------------------------- FP8
@pytest.mark.parametrize("m", [1, 2048])
def test_fp8_linear_matches_fp64_oracle(m, gemm_path):
    """BASELINE config 4 (A bf16 -> e4m3 per token, W e4m3 per channel, bf16
    out; K = N = 5120, plus the M = 1 decode shape).  Codes bit-exact; every
    output within 1 bf16 ulp plus the fp32 accumulation term 2^-20 * sum|a*w|
    of the exact e4m3 products."""
    rng = np.random.default_rng(20261108 + m)
    n = k = 5120
    xt = x_tensor(rng.standard_normal((m, k)).astype(np.float32), torch.bfloat16)
    w = torch.from_numpy((rng.standard_normal((n, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, quant="e4m3")
    y = rdna2_ops.fp8_linear(xt, wq, sw, out_dtype=torch.bfloat16)
    aq, sa = oracle.quant_rows_e4m3(oracle.decode(bits(xt), oracle.BF16))
    qa, _ = rdna2_ops.act_quant(xt, quant="e4m3")
    assert np.array_equal(qa.view(torch.uint8).cpu().numpy(), aq)
    a64 = oracle.decode_e4m3(aq).astype(np.float64)
    w64 = oracle.decode_e4m3(wq.view(torch.uint8).cpu().numpy()).astype(np.float64)
    scale = sa.astype(np.float64)[:, None] * sw.cpu().numpy().astype(np.float64)[None, :]
    ref = (a64 @ w64.T) * scale
    absref = (np.abs(a64) @ np.abs(w64).T) * scale
    got = oracle.decode(bits(y), oracle.BF16)
    assert_within_ulp(got, ref, absref, "bf16", f"fp8 config4 M={m} {gemm_path}")
