"""FP8 weight GEMM surface on the GPU (reference rdna2_ops/fp8_weight_gemm_v06.py).

* decode: exhaustive 256-pattern check of bench_dtype_gemm_v06.py:232-245
  (finite bits equal to torch's native cast, NaN and +-Inf classes equal);
* int8 methods: reference row quantizer (_quant_rows) codes/scales bit-exact,
  INT32 GEMM exact, fp32 epilogue bit-exact, cast to fp16;
* float methods and scaled e4m3: every output within 1 ulp of the output
  type plus the fp32 accumulation term 2^-20 * sum|a*w| (exact products,
  fp32 accumulation in tensor-core order; conftest.assert_within_ulp)."""
import numpy as np
import pytest

import oracle
from conftest import assert_within_ulp

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import fp8_weight_gemm_v06 as f8  # noqa: E402


@pytest.fixture(autouse=True, scope="module")
def _status():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0


def _bits16(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_decode_all_256_patterns(dtype, out_dtype):
    raw = torch.arange(256, device="cuda", dtype=torch.int16).to(torch.uint8).reshape(16, 16)
    fp8 = raw.view(dtype)
    native = fp8.to(out_dtype)
    meta = {}
    cand = f8.decode_fp8_weight(fp8, out_dtype=out_dtype, metadata=meta)
    fin = torch.isfinite(native)
    iv = torch.int16 if out_dtype == torch.float16 else torch.int32
    assert torch.equal(native[fin].view(iv), cand[fin].view(iv))
    assert torch.equal(torch.isnan(native), torch.isnan(cand))
    assert torch.equal(torch.isposinf(native), torch.isposinf(cand))
    assert torch.equal(torch.isneginf(native), torch.isneginf(cand))
    assert meta["method"] == "software_decode"


def _fp8_weight(seed, n, k, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn((n, k), generator=g, device="cuda") / np.sqrt(k)).to(torch.bfloat16).to(dtype)


def _decoded(w):
    codes = w.view(torch.uint8).cpu().numpy()
    return oracle.decode_e4m3(codes) if w.dtype == torch.float8_e4m3fn else oracle.decode_e5m2(codes)


@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_prepare_int8_weight_matches_reference_quantizer(dtype):
    w = _fp8_weight(20261108, 300, 1000, dtype)
    qw, sw = f8.prepare_int8_weight(w)
    rq, rs = oracle.quant_rows_ref(_decoded(w))
    assert np.array_equal(qw.cpu().numpy(), rq)
    assert np.array_equal(sw.cpu().numpy().view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("method", ["int8", "prepared_int8"])
@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_int8_methods_bit_exact(method, dtype):
    m, n, k = 190, 520, 1024
    w = _fp8_weight(1, n, k, dtype)
    a = (torch.randn((m, k), device="cuda") * 0.25).half()
    bias = (torch.randn(n, device="cuda") * 0.05).half()
    prep = f8.prepare_int8_weight(w) if method == "prepared_int8" else None
    y = f8.fp8_weight_gemm(a, w, bias=bias, method=method, prepared=prep)
    qa, sa = oracle.quant_rows_ref(oracle.decode(_bits16(a), oracle.F16))
    qw, sw = oracle.quant_rows_ref(_decoded(w))
    acc = oracle.gemm_s8(qa, qw)
    y32 = oracle.epilogue_s32(acc, sa, sw, _bits16(bias), oracle.F16, oracle.EPI_SEPARATE, oracle.F32)
    assert np.array_equal(_bits16(y), oracle.encode(y32, oracle.F16))


@pytest.mark.parametrize("method", ["upcast", "decode", "fused_dot2", "prepared_fp16"])
def test_float_methods(method):
    m, n, k = 130, 384, 768
    w = _fp8_weight(2, n, k, torch.float8_e4m3fn)
    a = (torch.randn((m, k), device="cuda") * 0.25).half()
    bias = (torch.randn(n, device="cuda") * 0.05).half()
    prep = w.half() if method == "prepared_fp16" else None
    y = f8.fp8_weight_gemm(a, w, bias=bias, method=method, prepared=prep)
    af = oracle.decode(_bits16(a), oracle.F16).astype(np.float64)
    wf = _decoded(w).astype(np.float64)
    ref = af @ wf.T + oracle.decode(_bits16(bias), oracle.F16).astype(np.float64)[None, :]
    absref = np.abs(af) @ np.abs(wf).T
    got = oracle.decode(_bits16(y), oracle.F16)
    assert_within_ulp(got, ref, absref, "fp16", method)


@pytest.mark.parametrize("m", [1, 2048])
def test_scaled_e4m3_method_config4(m):
    """BASELINE config 4 through the reference-named entry point
    fp8_weight_gemm(method="scaled_e4m3"): activation codes bit-exact with the
    oracle's per-token e4m3 quantizer, and every output within 1 bf16 ulp
    plus the fp32 accumulation term of the exact f64 value."""
    n = k = 5120
    gen = torch.Generator(device="cuda").manual_seed(20261108 + m)
    a = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
    wf = torch.randn((n, k), generator=gen, device="cuda") * 0.02
    wq, sw = f8.prepare_scaled_e4m3_weight(wf)
    y = f8.fp8_weight_gemm(a, wq, method="scaled_e4m3", w_scale=sw)
    assert y.dtype == torch.bfloat16 and y.shape == (m, n)
    aq, sa = oracle.quant_rows_e4m3(oracle.decode(_bits16(a), oracle.BF16))
    rq, rs = oracle.quant_rows_e4m3(wf.cpu().numpy())
    assert np.array_equal(wq.view(torch.uint8).cpu().numpy(), rq)
    assert np.array_equal(sw.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    a64 = oracle.decode_e4m3(aq).astype(np.float64)
    w64 = oracle.decode_e4m3(rq).astype(np.float64)
    scale = sa.astype(np.float64)[:, None] * rs.astype(np.float64)[None, :]
    ref = (a64 @ w64.T) * scale
    absref = (np.abs(a64) @ np.abs(w64).T) * scale
    assert_within_ulp(oracle.decode(_bits16(y), oracle.BF16), ref, absref, "bf16", f"scaled_e4m3 M={m}")


def test_rejects_bad_calls():
    w = _fp8_weight(3, 64, 128, torch.float8_e4m3fn)
    with pytest.raises(ValueError):
        f8.fp8_weight_gemm(torch.zeros((4, 128), device="cuda", dtype=torch.float32), w)
    with pytest.raises(ValueError):
        f8.fp8_weight_gemm(torch.zeros((4, 128), device="cuda", dtype=torch.float16), w, method="nope")
    with pytest.raises(TypeError):
        f8.decode_fp8_weight(torch.zeros((4, 4), device="cuda"))
