"""INT4 path on the GPU: device packer/decoder bit-exact against the
reference's pack_int4_cpu golden vectors, and the tcgen05 W4A16 GEMM against
the fp64 CPU oracle at every BASELINE config-3 token count.

W4A16 tolerance: the dequantized 16-bit weights are bit-exact by
construction; the GEMM accumulates exact fp32 products in an order the
tensor core chooses, so every output must lie within 1 ulp of the 16-bit
output type plus the fp32 accumulation term 2^-20 * sum|a*w|
(conftest.assert_within_ulp), checked on every output of every shape."""
import numpy as np
import pytest

import oracle
from conftest import assert_within_ulp

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import int4_weight_gemm_v07 as i4  # noqa: E402

ODT = {torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}


@pytest.fixture(autouse=True, scope="module")
def _status():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("order", ["low", "high"])
def test_pack_int4_matches_reference_golden(golden, g, sym, layout, order):
    """Device packer == reference pack_int4_cpu on bench_int4_v07.py:85-95's
    smoke weights (zero row, full nibble ranges) for every combination."""
    z = golden("int4_packing.npz")
    key = f"g{g}_{'sym' if sym else 'aff'}_{layout}_{order}"
    w = torch.from_numpy(z["w"]).cuda()
    p = i4.pack_int4(w, group_size=g, symmetric=sym, layout=layout, order=order)
    for f in ("data", "scales", "zeros", "sums"):
        got = getattr(p, f).cpu().numpy()
        ref = z[key + "_" + f]
        assert got.dtype == ref.dtype and np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f
    assert np.array_equal(i4.unpack_int4(p, dtype=torch.int8).cpu().numpy().astype(np.int32),
                          z[key + "_centered"])
    assert np.array_equal(i4.unpack_int4(p, dtype=torch.float32).cpu().numpy().view(np.uint32),
                          z[key + "_float"].view(np.uint32))


def _tiles_cpu(p, dtype):
    """numpy restatement of the W4A16 tile format (include/b2_qlinear.h):
    u = q + 8 with element j of a word at nibble (j >> 1) + 4*(j & 1), 4 KiB
    chunks [T][K/64][128][8]; group words {16-bit scale, zu} [T][G][128]."""
    words = p.data.cpu().numpy().view(np.uint32)
    if p.layout == "kn":
        words = words.T
    words = np.ascontiguousarray(words).astype(np.uint64)
    shifts = np.arange(8, dtype=np.uint64) * 4
    if p.order == "high":
        shifts = 28 - shifts
    nib = ((words[..., None] >> shifts) & 15) ^ 8                      # [N, K/8, 8] = u
    pos = np.array([(j >> 1) + 4 * (j & 1) for j in range(8)], dtype=np.uint64) * 4
    inter = (nib << pos).sum(-1).astype(np.uint32)                      # [N, K/8]
    t = -(-p.n // 128)
    pad = np.zeros((t * 128, p.k // 8), np.uint32)
    pad[:p.n] = inter
    tiles = pad.reshape(t, 128, p.k // 64, 8).transpose(0, 2, 1, 3)
    s16 = p.scales.cpu().to(dtype).view(torch.int16).numpy().view(np.uint16).astype(np.uint32)
    z16 = (p.zeros.cpu() + 8).to(dtype).view(torch.int16).numpy().view(np.uint16).astype(np.uint32)
    g = p.k // p.group_size
    grp = np.zeros((t * 128, g), np.uint32)
    grp[:p.n] = s16 | (z16 << 16)
    return np.ascontiguousarray(tiles), np.ascontiguousarray(grp.reshape(t, 128, g).transpose(0, 2, 1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("order", ["low", "high"])
def test_prepare_w4a16_tiles_bit_exact(golden, dtype, g, layout, order):
    """b2_w4a16_prepare == the numpy restatement, from the reference's golden
    packs of every layout / nibble order (zero rows and full nibble ranges)."""
    z = golden("int4_packing.npz")
    key = f"g{g}_aff_{layout}_{order}"
    n, k = z["w"].shape
    if k % 64:
        pytest.skip("W4A16 tiles need K % 64 == 0")
    p = i4.PackedInt4(*(torch.from_numpy(z[key + "_" + f]) for f in ("data", "scales", "zeros", "sums")),
                      n, k, g, False, layout, order)
    wt = i4.prepare_w4a16(p.to("cuda"), dtype)
    tiles, grp = _tiles_cpu(p, dtype)
    assert np.array_equal(wt.tiles.cpu().numpy().view(np.uint32), tiles)
    assert np.array_equal(wt.groups.cpu().numpy().view(np.uint32), grp)


def _ref_w4a16(a_bits, a_code, p_cpu, dtype):
    """fp64 oracle: bf16/fp16-rounded scales, w = round((u - zu) * s), fp64 dot."""
    s16 = p_cpu.scales.to(dtype).float().numpy()
    w = oracle.dequant_int4(p_cpu.data.numpy(), s16, p_cpu.zeros.float().numpy(), p_cpu.group_size,
                            out_dtype=ODT[dtype])
    a = oracle.decode(a_bits, a_code).astype(np.float64)
    w = w.astype(np.float64)
    return a @ w.T, np.abs(a) @ np.abs(w).T


def _bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def _check(y, ref, absref, dtype, bias=None, what="w4a16"):
    got = oracle.decode(_bits(y), ODT[dtype]).astype(np.float64)
    if bias is not None:
        ref = ref + oracle.decode(_bits(bias), ODT[dtype]).astype(np.float64)[None, :]
    assert_within_ulp(got, ref, absref, "bf16" if dtype == torch.bfloat16 else "fp16", what)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k,g", [(17, 19, 384, 32), (17, 19, 384, 64), (17, 19, 384, 128),
                                     (33, 300, 1024, 128), (200, 520, 512, 64)])
def test_w4a16_small_shapes(dtype, m, n, k, g):
    gen = torch.Generator().manual_seed(20261107 + m + n)
    w = torch.randn((n, k), generator=gen) * 0.2
    w[0] = 0
    p_cpu = i4.pack_int4_cpu(w, group_size=g, symmetric=False)
    a = (torch.randn((m, k), generator=gen) * 0.5).to(dtype)
    bias = (torch.randn(n, generator=gen) * 0.1).to(dtype)
    y = i4.int4_linear_a16(a.cuda(), p_cpu.to("cuda"), bias=bias.cuda())
    ref, absref = _ref_w4a16(_bits(a), ODT[dtype], p_cpu, dtype)
    _check(y, ref, absref, dtype, bias)


@pytest.fixture(params=["tmem", "smem"])
def w4_path(request):
    i4.set_w4a16_path(request.param)
    yield request.param
    i4.set_w4a16_path("auto")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 16, 17, 40, 64, 100, 128, 129, 300])
@pytest.mark.parametrize("g", [32, 128])
def test_w4a16_schedules(dtype, m, g, w4_path):
    """Stream-K (M <= 128: a CTA's range crosses tiles, group stages start
    mid-group) and whole-tile (M > 128, ragged token and row tiles) runs
    against the oracle; N = 1000 leaves a partial last row tile."""
    n, k = 1000, 1152
    gen = torch.Generator().manual_seed(20261108 + m + g)
    w = torch.randn((n, k), generator=gen) * 0.05
    p_cpu = i4.pack_int4_cpu(w, group_size=g, symmetric=False)
    a = torch.randn((m, k), generator=gen).to(dtype)
    bias = (torch.randn(n, generator=gen) * 0.1).to(dtype)
    y = i4.int4_linear_a16(a.cuda(), p_cpu.to("cuda"), bias=bias.cuda())
    ref, absref = _ref_w4a16(_bits(a), ODT[dtype], p_cpu, dtype)
    _check(y, ref, absref, dtype, bias)


@pytest.fixture(scope="module")
def config3_pack():
    """BASELINE config 3 weight: W [14336,4096] ~ N(0,0.02), affine uint4 g128,
    packed on the CPU by pack_int4_cpu (the packer the reference goldens pin);
    the device packer must produce the same pack."""
    n, k = 14336, 4096
    gen = torch.Generator().manual_seed(20261107)
    w = torch.randn((n, k), generator=gen) * 0.02
    p_cpu = i4.pack_int4_cpu(w, group_size=128, symmetric=False)
    p_dev = i4.pack_int4(w.cuda(), group_size=128, symmetric=False)
    for f in ("data", "scales", "zeros", "sums"):
        assert torch.equal(getattr(p_dev, f).cpu().view(torch.int32), getattr(p_cpu, f).view(torch.int32)), f
    return p_cpu, i4.prepare_w4a16(p_cpu.to("cuda"), torch.bfloat16)


@pytest.mark.parametrize("m", [1, 16, 128, 2048])
def test_w4a16_config3(m, config3_pack, w4_path):
    """bf16 A [M,4096] ~ N(0,1) against the CPU-packed
    weight, bf16 out; every one of the M x 14336 outputs checked."""
    dtype = torch.bfloat16
    p_cpu, wt = config3_pack
    gen = torch.Generator().manual_seed(20261107 + m)
    a = torch.randn((m, p_cpu.k), generator=gen).to(dtype)
    y = i4.w4a16_gemm(a.cuda(), wt)
    ref, absref = _ref_w4a16(_bits(a), ODT[dtype], p_cpu, dtype)
    _check(y, ref, absref, dtype, what=f"config3 M={m}")


def test_w4a16_deterministic_split_k(w4_path):
    dtype = torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(3)
    w = torch.randn((4096, 4096), generator=gen, device="cuda") * 0.02
    wt = i4.quantize_w4a16(w, group_size=128, dtype=dtype)
    a = torch.randn((8, 4096), generator=gen, device="cuda").to(dtype)
    assert nat.library().b2_w4a16_workspace_bytes(8, 4096, 4096, 128) > 0  # stream-K slots engaged
    y1, y2 = i4.w4a16_gemm(a, wt), i4.w4a16_gemm(a, wt)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_dense_linear_kind_f16(dtype):
    gen = torch.Generator().manual_seed(8)
    m, n, k = 300, 520, 1024
    a = torch.randn((m, k), generator=gen).to(dtype)
    w = (torch.randn((n, k), generator=gen) * 0.05).to(dtype)
    y = i4.dense_linear(a.cuda(), w.cuda())
    af, wf = oracle.decode(_bits(a), ODT[dtype]), oracle.decode(_bits(w), ODT[dtype])
    _check(y, oracle.gemm_f32_f64(af, wf), oracle.gemm_f32_f64(np.abs(af), np.abs(wf)), dtype)


def test_w4a16_workspace_reuse_leaves_counters_zero():
    """One caller-owned workspace across decode calls of different shapes:
    results equal fresh-workspace calls bit for bit, and the arrival
    counters at its end are zero again after every call."""
    dtype = torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(11)
    shapes = [(8, 4096, 2048), (1, 1000, 1152), (32, 2304, 4096), (8, 4096, 2048)]
    lib = nat.library()
    need = max(lib.b2_w4a16_workspace_bytes(m, n, k, 128) for m, n, k in shapes)
    ws = torch.zeros(need, device="cuda", dtype=torch.uint8)
    for m, n, k in shapes:
        w = torch.randn((n, k), generator=gen, device="cuda") * 0.02
        wt = i4.quantize_w4a16(w, group_size=128, dtype=dtype)
        a = torch.randn((m, k), generator=gen, device="cuda").to(dtype)
        y_shared = i4.w4a16_gemm(a, wt, workspace=ws)
        y_fresh = i4.w4a16_gemm(a, wt)
        assert torch.equal(y_shared.view(torch.int16), y_fresh.view(torch.int16))
        assert int(ws[:4096].count_nonzero()) == 0  # the arrival counters


# ------------------------------------------------------------------ W4A8
def _packed_from_golden(z, key, n, k, g, layout, order):
    f = {name: torch.from_numpy(z[key + "_" + name]) for name in ("data", "scales", "zeros", "sums")}
    return i4.PackedInt4(f["data"], f["scales"], f["zeros"], f["sums"], n, k, g, False, layout, order).to("cuda")


def test_w4a8_matches_reference_grouped_output(golden):
    """int4_linear_a8 reproduces the reference's grouped_integer_reference
    output (int4_model_switches_v07.py:19-34) bit for bit: g32 affine kn
    pack, per-row scales, bias."""
    z = golden("int4_packing.npz")
    n, k = z["grouped_w"].shape
    p = i4.PackedInt4(torch.from_numpy(z["grouped_data"]), torch.from_numpy(z["grouped_scales"]),
                      torch.from_numpy(z["grouped_zeros"]), torch.zeros_like(torch.from_numpy(z["grouped_zeros"])),
                      n, k, 32, False, "kn", "low").to("cuda")
    a = torch.from_numpy(z["grouped_a"]).cuda()
    sa = torch.from_numpy(z["grouped_sa"]).cuda()
    bias = torch.from_numpy(z["grouped_bias"]).cuda()
    y = i4.int4_linear_a8(a, p, sa, bias=bias)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), z["grouped_y"].view(np.uint32))


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("order", ["low", "high"])
def test_w4a8_integer_mode_matches_int_oracle(golden, g, sym, layout, order):
    z = golden("int4_packing.npz")
    key = f"g{g}_{'sym' if sym else 'aff'}_{layout}_{order}"
    n, k = z["w"].shape
    p = _packed_from_golden(z, key, n, k, g, layout, order)
    a = torch.from_numpy(z["a"]).cuda()
    y = i4.int4_linear_a8(a, p, None, integer=True)
    assert np.array_equal(y.cpu().numpy().astype(np.int64), z[key + "_int_oracle"])


@pytest.mark.parametrize("m", [1, 5, 16, 17, 33, 64, 100, 200])
@pytest.mark.parametrize("g", [32, 64, 128])
def test_w4a8_random_shapes_bit_exact(m, g):
    """Ragged N (partial last row tile), token tiles 16/32/64 and several
    token tiles, every group size: bit-exact against the oracle."""
    n, k = 1000, 1152
    gen = torch.Generator().manual_seed(20261105 + m + g)
    w = torch.randn((n, k), generator=gen) * 0.05
    p_cpu = i4.pack_int4_cpu(w, group_size=g, symmetric=False)
    a = torch.randint(-128, 128, (m, k), generator=gen, dtype=torch.int8)
    sa = torch.rand(m, generator=gen) * 0.02 + 0.001
    bias = torch.randn(n, generator=gen) * 0.01
    wt = i4.prepare_w4a8(p_cpu.to("cuda"))
    y = i4.int4_linear_a8(a.cuda(), None, sa.cuda(), bias=bias.cuda(), prepared=wt)
    c = i4.unpack_int4_cpu(p_cpu, floating=False).numpy().astype(np.int8)
    ref = oracle.w4a8_linear(a.numpy(), c, p_cpu.scales.numpy(), g, sa.numpy(), bias.numpy())
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
