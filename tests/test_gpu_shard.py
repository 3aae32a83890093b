"""The column-parallel INT8 activation exchange (b2_shard_amax +
b2_shard_codes) and the gathered GEMM on codes (b2_qgemm_gather) on ONE
GPU: P "virtual ranks" share one stream, each rank's peer buffers being
other buffers of the same device.  Every phase of every rank is enqueued
before any wait that needs it, so no kernel waits on a later kernel.  The
codes and scales every rank ends with must equal the whole-row activation
prologue (b2_act_quant) on the next layer's input bit for bit."""
import ctypes

import numpy as np
import pytest

from conftest import outlier_activations

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rdna2_ops  # noqa: E402
from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import qlinear  # noqa: E402
from rdna2_ops.column_parallel import shard_overlap  # noqa: E402


@pytest.fixture(autouse=True, scope="module")
def _status():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0


def _arr(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


class VirtualExchange:
    def __init__(self, world, m, ldq):
        sb = nat.library().b2_gather_state_bytes()
        self.world, self.m, self.ldq = world, m, ldq
        self.xchg = [torch.full((world * m,), float("nan"), device="cuda") for _ in range(world)]
        self.codes = [torch.zeros((m, ldq), device="cuda", dtype=torch.int8) for _ in range(world)]
        self.scale = [torch.full((m,), float("nan"), device="cuda") for _ in range(world)]
        self.st_a = [torch.zeros(sb, device="cuda", dtype=torch.uint8) for _ in range(world)]
        self.st_c = [torch.zeros(sb, device="cuda", dtype=torch.uint8) for _ in range(world)]
        self.xchg_p = _arr([t.data_ptr() for t in self.xchg])
        self.codes_p = _arr([t.data_ptr() for t in self.codes])
        self.st_a_p = _arr([t.data_ptr() for t in self.st_a])
        self.st_c_p = _arr([t.data_ptr() for t in self.st_c])


def _exchange(vx, slices, lo, block, dtype, epoch, quant=0):
    """slices[r] = (tensor [m, width] view of rank r's slice, width, col0)."""
    lib = nat.library()
    s = nat.stream_ptr(torch.device("cuda"))
    code = nat.DTYPE_CODE[dtype]
    for r, (y, width, col0) in enumerate(slices):
        ldy = y.stride(0) if width else 64
        nat.check(lib.b2_shard_amax(y.data_ptr(), code, vx.m, width, ldy, block, vx.world, r, vx.xchg_p,
                                    vx.st_a_p, epoch, s), "b2_shard_amax")
    for r, (y, width, col0) in enumerate(slices):
        ldy = y.stride(0) if width else 64
        nat.check(lib.b2_gather_wait(vx.st_a[r].data_ptr(), vx.world, epoch, s), "b2_gather_wait")
        nat.check(lib.b2_shard_codes(y.data_ptr(), code, vx.m, width, ldy, block, quant, vx.world, r,
                                     vx.xchg[r].data_ptr(), vx.codes_p, vx.ldq, col0, vx.scale[r].data_ptr(),
                                     vx.st_c_p, epoch, s), "b2_shard_codes")
    for r in range(vx.world):
        nat.check(lib.b2_gather_wait(vx.st_c[r].data_ptr(), vx.world, epoch, s), "b2_gather_wait")


CASES = [  # world, shard width, next-input range [lo, hi), block, dtype, M
    (1, 1536, 0, 1536, 128, torch.float16, 300),
    (2, 768, 0, 512, 128, torch.float16, 300),       # rank 1 holds none of the range
    (3, 1152, 0, 3072, 128, torch.float16, 1000),    # QKV -> Q third: the last rank holds part of it
    (4, 512, 512, 2048, 256, torch.bfloat16, 77),    # rank 0 before the range
    (8, 1536, 0, 12288, 128, torch.float16, 513),
    (8, 384, 0, 3072, 0, torch.float32, 64),         # no rotation
    (2, 6144, 0, 12288, 2048, torch.float16, 40),    # 32-lane rotation blocks
]


@pytest.mark.parametrize("world,ns,lo,hi,block,dtype,m", CASES)
def test_shard_codes_equal_whole_row_prologue(world, ns, lo, hi, block, dtype, m):
    rng = np.random.default_rng(world * 131 + m)
    n_total = world * ns
    y_full = torch.from_numpy(outlier_activations(rng, m, n_total)).to(dtype).cuda()
    ref_q, ref_s = qlinear.act_quant(y_full[:, lo:hi], rotation_block=block or None)
    ldq = -(-(hi - lo) // 16) * 16
    vx = VirtualExchange(world, m, ldq)
    ys = [y_full[:, r * ns:(r + 1) * ns].contiguous() for r in range(world)]
    for epoch in (1, 2):                                   # the states and buffers are reused
        for t in vx.codes:
            t.fill_(0x55)
        slices = []
        for r in range(world):
            a, b = shard_overlap(r * ns, ns, lo, hi)
            slices.append((ys[r][:, a - r * ns:] if b > a else ys[r], b - a, a - lo))
        _exchange(vx, slices, lo, block, dtype, epoch)
        torch.cuda.synchronize()
        for r in range(world):
            assert torch.equal(vx.codes[r][:, :hi - lo], ref_q), (epoch, r)
            assert torch.equal(vx.scale[r].view(torch.int32), ref_s.view(torch.int32)), (epoch, r)
    for st in vx.st_a + vx.st_c:
        words = st.view(torch.int32).cpu().numpy()
        assert list(words[:world]) == [2] * world and words[32] == 0
    assert nat.device_status() == 0


def test_shard_codes_e4m3_equal_whole_row_prologue():
    world, ns, m = 4, 768, 200
    rng = np.random.default_rng(5)
    y_full = torch.from_numpy(outlier_activations(rng, m, world * ns)).half().cuda()
    ref_q, ref_s = qlinear.act_quant(y_full, rotation_block=128, quant="e4m3")
    vx = VirtualExchange(world, m, world * ns)
    slices = [(y_full[:, r * ns:(r + 1) * ns], ns, r * ns) for r in range(world)]   # strided slices in place
    _exchange(vx, slices, 0, 128, torch.float16, 1, quant=1)
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(vx.codes[r].view(torch.uint8), ref_q.view(torch.uint8)), r
        assert torch.equal(vx.scale[r].view(torch.int32), ref_s.view(torch.int32)), r


def test_qgemm_gather_equals_single_gpu_gemm():
    """Codes in, fp16 Y gathered to every virtual rank: equals b2_qgemm on
    the whole weight."""
    world, m, n_total, k = 4, 700, 2048, 1024
    rng = np.random.default_rng(9)
    x = torch.from_numpy(outlier_activations(rng, m, k)).half().cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, rotation_block=128)
    q, sa = qlinear.act_quant(x, rotation_block=128)
    ref = rdna2_ops.w8a8_linear(x, wq, sw, rotation_block=128, out_dtype=torch.float16)
    lib = nat.library()
    outs = [torch.full((m, n_total), float("nan"), device="cuda", dtype=torch.float16) for _ in range(world)]
    states = [torch.zeros(lib.b2_gather_state_bytes(), device="cuda", dtype=torch.uint8) for _ in range(world)]
    op, sp = _arr([t.data_ptr() for t in outs]), _arr([t.data_ptr() for t in states])
    ns = n_total // world
    s = nat.stream_ptr(x.device)
    shards = [(wq[r * ns:(r + 1) * ns].contiguous(), sw[r * ns:(r + 1) * ns].contiguous()) for r in range(world)]
    for r, (wr, swr) in enumerate(shards):
        nat.check(lib.b2_qgemm_gather(nat.KIND_I8, q.data_ptr(), k, sa.data_ptr(), wr.data_ptr(), k, m, ns, k,
                                      swr.data_ptr(), ns, None, 0, nat.EPI_SEPARATE, nat.F16, n_total, r * ns,
                                      world, r, op, sp, 1, s), "b2_qgemm_gather")
    for r in range(world):
        nat.check(lib.b2_gather_wait(states[r].data_ptr(), world, 1, s), "b2_gather_wait")
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(outs[r].view(torch.int16), ref.view(torch.int16)), r


def test_shard_rejects_bad_calls():
    lib = nat.library()
    vx = VirtualExchange(2, 64, 256)
    y = torch.zeros((64, 256), device="cuda", dtype=torch.float16)
    args = (y.data_ptr(), nat.F16, 64)
    assert lib.b2_shard_amax(*args, 96, 256, 128, 2, 0, vx.xchg_p, vx.st_a_p, 1, None) != 0   # width % 64
    assert lib.b2_shard_amax(*args, 128, 256, 128, 2, 0, vx.xchg_p, vx.st_a_p, 0, None) != 0  # epoch 0
    assert lib.b2_shard_amax(*args, 192, 256, 128, 2, 0, vx.xchg_p, vx.st_a_p, 1, None) != 0  # width % block
    assert lib.b2_shard_amax(*args, 128, 256, 128, 2, 2, vx.xchg_p, vx.st_a_p, 1, None) != 0  # rank
    assert lib.b2_shard_codes(*args, 128, 256, 128, 0, 2, 0, vx.xchg[0].data_ptr(), vx.codes_p, 256, 136,
                              vx.scale[0].data_ptr(), vx.st_c_p, 1, None) != 0                 # col0 + width
    assert lib.b2_shard_codes(*args, 128, 256, 128, 0, 2, 0, vx.xchg[0].data_ptr(), vx.codes_p, 256, 8,
                              vx.scale[0].data_ptr(), vx.st_c_p, 1, None) != 0                 # col0 % 16
    assert lib.b2_shard_codes(*args, 128, 256, 128, 3, 2, 0, vx.xchg[0].data_ptr(), vx.codes_p, 256, 0,
                              vx.scale[0].data_ptr(), vx.st_c_p, 1, None) != 0                 # quant
    torch.cuda.synchronize()


@pytest.mark.parametrize("ns,lo,hi,block,dtype,m", [(1536, 0, 1536, 128, torch.float16, 300),
                                                    (3072, 0, 1024, 256, torch.bfloat16, 77),
                                                    (12288, 0, 12288, 128, torch.float16, 513)])
def test_shard_exchange_fused_one_rank(ns, lo, hi, block, dtype, m):
    """The one-launch exchange (absmax pass, in-kernel barrier, codes pass)
    on a single rank -- the only form one GPU may run, since ranks sharing a
    device would wait on each other inside their kernels -- equals the
    whole-row prologue bit for bit over two calls."""
    rng = np.random.default_rng(ns + m)
    y = torch.from_numpy(outlier_activations(rng, m, ns)).to(dtype).cuda()
    ref_q, ref_s = qlinear.act_quant(y[:, lo:hi], rotation_block=block)
    ldq = -(-(hi - lo) // 16) * 16
    vx = VirtualExchange(1, m, ldq)
    lib = nat.library()
    for epoch in (1, 2):
        vx.codes[0].fill_(0x55)
        nat.check(lib.b2_shard_exchange(y[:, lo:].data_ptr(), nat.DTYPE_CODE[dtype], m, hi - lo, ns, block, 0, 1, 0,
                                        vx.xchg_p, vx.st_a_p, epoch, vx.codes_p, ldq, 0, vx.scale[0].data_ptr(),
                                        vx.st_c_p, epoch, nat.stream_ptr(y.device)), "b2_shard_exchange")
        nat.check(lib.b2_gather_wait(vx.st_c[0].data_ptr(), 1, epoch, nat.stream_ptr(y.device)), "b2_gather_wait")
        torch.cuda.synchronize()
        assert torch.equal(vx.codes[0][:, :hi - lo], ref_q), epoch
        assert torch.equal(vx.scale[0].view(torch.int32), ref_s.view(torch.int32)), epoch
    assert nat.device_status() == 0


def test_shard_exchange_barrier_gives_up_when_a_rank_never_comes():
    """Rank 0 of two runs the one-launch exchange; rank 1 never does, so its
    absmax slots never arrive.  Every CTA's in-kernel wait ends after its
    2 s bound with status 0x107, no codes phase runs and nothing is
    released; the context still runs a linear afterwards."""
    nat.device_status(reset=True)
    lib = nat.library()
    m, ns = 64, 256
    vx = VirtualExchange(2, m, 2 * ns)
    y = torch.ones((m, ns), device="cuda", dtype=torch.float16)
    nat.check(lib.b2_shard_exchange(y.data_ptr(), nat.F16, m, ns, ns, 128, 0, 2, 0, vx.xchg_p, vx.st_a_p, 1,
                                    vx.codes_p, 2 * ns, 0, vx.scale[0].data_ptr(), vx.st_c_p, 1,
                                    nat.stream_ptr(y.device)), "b2_shard_exchange")
    torch.cuda.synchronize()
    assert nat.device_status(reset=True) == 0x107
    assert int(vx.st_c[1].view(torch.int32)[0]) == 0            # no codes released to the other rank
    assert torch.isfinite(rdna2_ops.w8a8_linear(y, torch.ones((64, ns), device="cuda", dtype=torch.int8),
                                                torch.ones(64, device="cuda"), out_dtype=torch.float32)).all()
    assert nat.device_status() == 0
