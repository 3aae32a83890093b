"""Pin the CPU oracle to the reference's own outputs (golden vectors) and to
the frozen rotation/quantizer contract.  CPU only."""
import numpy as np
import pytest

import oracle
from conftest import outlier_activations


# ------------------------------------------------------------------ codecs
def test_f16_bf16_codecs_match_numpy_and_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000).astype(np.float32)
         * (10.0 ** rng.integers(-9, 6, 100000)).astype(np.float32))
    x = np.concatenate([x, np.array([0.0, -0.0, 65504, 65520, 1e-8, 5.96e-8, np.inf, -np.inf],
                                    np.float32)])
    with np.errstate(over="ignore"):
        assert np.array_equal(oracle.encode(x, oracle.F16), x.astype(np.float16).view(np.uint16))
    tb = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.encode(x, oracle.BF16), tb)
    allh = np.arange(65536, dtype=np.uint16)
    d, ref = oracle.decode(allh, oracle.F16), allh.view(np.float16).astype(np.float32)
    assert np.all((d.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(d) & np.isnan(ref)))


def test_e4m3_decode_all_256_patterns(golden):
    """Exhaustive decode check of bench_dtype_gemm_v06.py:232-245 (finite bits,
    NaN class) against torch's native float8_e4m3fn cast."""
    g = golden("fp8_decode.npz")
    dec = oracle.decode_e4m3(g["codes"])
    ref = g["e4m3"]
    fin = np.isfinite(ref)
    assert np.array_equal(dec[fin].view(np.uint32), ref[fin].view(np.uint32))
    assert np.array_equal(np.isnan(dec), np.isnan(ref))


def test_e4m3_encode_rne_and_saturation():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(50000) * 10.0 ** rng.integers(-4, 3, 50000)).astype(np.float32)
    x = x[np.abs(x) <= 448]
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(oracle.encode_e4m3(x), ref)
    sat = oracle.encode_e4m3(np.array([449, 464, 1e30, -1e30], np.float32))
    assert list(sat) == [0x7E, 0x7E, 0x7E, 0xFE]


# --------------------------------------------------------------- INT8 path
@pytest.mark.parametrize("key", ["weight_nk_vector", "weight_nk_scalar", "rhs_kn_vector",
                                 "rhs_kn_scalar"])
def test_int8_known_answer(golden, key):
    """bench_int8_gemm.py:181-203: offset/padded A view, both B layouts, scalar
    and vector scales, bias; INT32 exact and FP32 epilogue bitwise."""
    g = golden("int8_known_answer.npz")
    a = g[key + "_a_store"][1:38, 1:80]
    acc = oracle.gemm_s8(a, g[key + "_w"])
    assert np.array_equal(acc, g[key + "_acc"])
    out = oracle.epilogue_s32(acc, g[key + "_sa"], g[key + "_sb"], g[key + "_bias"], oracle.F32,
                              oracle.EPI_SEPARATE, oracle.F32)
    assert np.array_equal(out.view(np.uint32), g[key + "_ref"].view(np.uint32))


@pytest.mark.parametrize("case", [0, 1, 2])
def test_moss_backend_epilogue(golden, case):
    """The reference backend.int8_linear (fp32 path, run with a stand-in Kitchen)
    equals the oracle's Kitchen epilogue bit for bit."""
    g = golden("moss_backend_fp32.npz")
    bias = g[f"c{case}_bias"] if f"c{case}_bias" in g.files else None
    y = oracle.w8a8_linear(g[f"c{case}_x"], oracle.F32, 0, g[f"c{case}_w"], g[f"c{case}_ws"],
                           bias, oracle.F32, oracle.EPI_KITCHEN, oracle.F32)
    assert np.array_equal(y.view(np.uint32), g[f"c{case}_y"].view(np.uint32))


def test_int32_accumulator_extremes():
    """|sum| reaches 128*128*K without overflow at the reference bound K=131071."""
    k = 131071
    a = np.full((2, k), -128, np.int8)
    w = np.full((3, k), -128, np.int8)
    w[1] = 127
    acc = oracle.gemm_s8(a, w)
    assert acc[0, 0] == 128 * 128 * k and acc[0, 1] == -128 * 127 * k


def test_quantizer_contract():
    x = np.array([[0.0] * 8, [1.0, -1.0, 0.5, 127 * 0.5 / 127, 2.0, -2.0, 0.0, 0.25],
                  [3.0, 1.5, -0.75, 0, 0, 0, 0, 0]], np.float32)
    q, s = oracle.quant_rows_int8(x)
    assert s[0] == 1.0 and not q[0].any()                     # zero row: scale 1, codes 0
    assert s[1] == np.float32(2.0) / np.float32(127.0)
    assert q[1, 4] == 127 and q[1, 5] == -127
    # ties go to even: x/s exactly k+0.5
    s2 = np.float32(3.0) / np.float32(127.0)
    xt = (np.array([0.5, 1.5, 2.5, -0.5, -2.5], np.float32) * s2).astype(np.float32)
    qt, _ = oracle.quant_rows_int8(np.concatenate([[3.0], xt]).astype(np.float32)[None])
    z = np.concatenate([[3.0], xt]).astype(np.float32) / s2
    assert np.array_equal(qt[0], np.clip(np.rint(z), -127, 127).astype(np.int8))


@pytest.mark.parametrize("block", [2, 8, 128, 256, 1024])
def test_rotation_is_orthonormal_block_hadamard(block):
    """fp32 FWHT == x @ blockdiag(H_B / sqrt(B)) (Sylvester H) within fp32 error,
    and the rotation preserves row norms."""
    rng = np.random.default_rng(block)
    k = max(2048, block * 2)
    x = outlier_activations(rng, 6, k)
    r = oracle.rotate_rows(x, oracle.F32, block)
    h = np.array([[1.0]])
    while h.shape[0] < block:
        h = np.block([[h, h], [h, -h]])
    ref = (x.astype(np.float64).reshape(6, k // block, block) @ (h / np.sqrt(block))).reshape(6, k)
    assert np.allclose(r, ref, rtol=1e-5, atol=1e-4 * np.abs(x).max())
    assert np.allclose(np.linalg.norm(r, axis=1), np.linalg.norm(x, axis=1), rtol=1e-5)


def test_rotation_identity_without_block():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 96)).astype(np.float32)
    assert np.array_equal(oracle.rotate_rows(x, oracle.F32, 0), x)


def test_rotated_linear_matches_unrotated_math():
    """Folding H into W: quantized rotated GEMM tracks the fp64 linear closely."""
    rng = np.random.default_rng(4)
    m, n, k = 64, 48, 512
    x = outlier_activations(rng, m, k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, 128))
    y = oracle.w8a8_linear(x, oracle.F32, 128, wq, sw, out_dtype=oracle.F32)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 0.02


# -------------------------------------------------------------------- INT4
@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("order", ["low", "high"])
def test_int4_packer_matches_pack_int4_cpu(golden, g, sym, order):
    """Restated packer == reference pack_int4_cpu on the bench_int4_v07.py:85-95
    smoke weights (zero row, full nibble ranges)."""
    z = golden("int4_packing.npz")
    key = f"g{g}_{'sym' if sym else 'aff'}_nk_{order}"
    p = oracle.pack_int4(z["w"], g, sym, order)
    for f in ("data", "scales", "zeros", "sums"):
        assert np.array_equal(p[f], z[key + "_" + f]), f
    kn = z[f"g{g}_{'sym' if sym else 'aff'}_kn_{order}_data"]
    assert np.array_equal(p["data"].T, kn)
    if order == "low":
        deq = oracle.dequant_int4(p["data"], p["scales"], p["zeros"].astype(np.float32), g,
                                  out_dtype=oracle.F32)
        assert np.array_equal(deq, z[key + "_float"])
        cen = z[key + "_centered"].astype(np.int64)
        assert np.array_equal(z["a"].astype(np.int64) @ cen.T, z[key + "_int_oracle"])


def test_int4_packer_baseline_format(golden):
    z = golden("int4_packing.npz")
    p = oracle.pack_int4(z["big_w"], 128, False, "low")
    for f in ("data", "scales", "zeros", "sums"):
        assert np.array_equal(p[f], z["big_" + f])


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("sym", [True, False])
def test_package_pack_int4_cpu_matches_golden(golden, g, sym):
    """The package's CPU packer (part of the reference API surface) equals the
    reference's pack_int4_cpu output on the smoke weights."""
    torch = pytest.importorskip("torch")
    from rdna2_ops.int4_weight_gemm_v07 import pack_int4_cpu, unpack_int4_cpu
    z = golden("int4_packing.npz")
    for layout in ("nk", "kn"):
        for order in ("low", "high"):
            key = f"g{g}_{'sym' if sym else 'aff'}_{layout}_{order}"
            p = pack_int4_cpu(torch.from_numpy(z["w"]), group_size=g, symmetric=sym, layout=layout,
                              order=order)
            for f in ("data", "scales", "zeros", "sums"):
                assert np.array_equal(getattr(p, f).numpy(), z[key + "_" + f]), (key, f)
            assert np.array_equal(unpack_int4_cpu(p, floating=False).numpy(), z[key + "_centered"])


def _centered(data, zeros, n, k, g, layout, order):
    """q - z from PackedInt4 storage (signed nibbles), numpy."""
    words = data.view(np.uint32) if layout == "nk" else data.view(np.uint32).T
    words = np.ascontiguousarray(words).astype(np.uint64)
    shifts = np.arange(8, dtype=np.uint64) * 4
    if order == "high":
        shifts = 28 - shifts
    q = ((words[..., None] >> shifts) & 15).astype(np.int32).reshape(n, k)
    q = np.where(q >= 8, q - 16, q)
    return (q - np.repeat(zeros, g, axis=1)).astype(np.int8)


def test_w4a8_oracle_matches_reference_grouped_integer_reference(golden):
    """The oracle's grouped W4A8 linear equals the reference's
    grouped_integer_reference output (int4_model_switches_v07.py:19-34) bit
    for bit (g32 affine "kn" pack, bias)."""
    z = golden("int4_packing.npz")
    a = z["grouped_a"]
    n, k = z["grouped_w"].shape
    c = _centered(z["grouped_data"], z["grouped_zeros"], n, k, 32, "kn", "low")
    y = oracle.w4a8_linear(a, c, z["grouped_scales"], 32, z["grouped_sa"], z["grouped_bias"])
    assert np.array_equal(y.view(np.uint32), z["grouped_y"].view(np.uint32))


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("order", ["low", "high"])
def test_w4a8_oracle_integer_mode_matches_int_oracle(golden, g, layout, order):
    z = golden("int4_packing.npz")
    key = f"g{g}_aff_{layout}_{order}"
    n, k = z["w"].shape
    c = _centered(z[key + "_data"], z[key + "_zeros"], n, k, g, layout, order)
    got = oracle.w4a8_linear(z["a"], c, z[key + "_scales"], g, np.ones(z["a"].shape[0], np.float32),
                             integer=True)
    assert np.array_equal(got.astype(np.int64), z[key + "_int_oracle"])
