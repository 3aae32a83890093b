"""The fused column-parallel gather (b2_quant_linear_gather + b2_gather_wait)
on ONE GPU: P "virtual ranks" run one after another on one stream, each
rank's peer buffers being other buffers of the same device.  Every peer
store (SM stores or TMA stores through per-peer tensor maps), flag slot, CTA count and bounded wait of the multi-GPU path runs as
it does across GPUs; only the IPC mapping is absent.  Every rank's full
output must equal the single-GPU fused linear of the whole weight bit for
bit (per-token scales see the whole row on every rank), over repeated
epochs, ragged M, every output dtype, both kinds, with and without bias.
No kernel here waits on another kernel: every wait is enqueued after all
the flags it needs were released."""
import ctypes

import numpy as np
import pytest

from conftest import outlier_activations

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rdna2_ops  # noqa: E402
from rdna2_ops import _native as nat  # noqa: E402
from rdna2_ops import qlinear  # noqa: E402

EPI = {"separate": nat.EPI_SEPARATE, "fused": nat.EPI_FMA, "kitchen": nat.EPI_KITCHEN}


@pytest.fixture(autouse=True, scope="module")
def _status():
    nat.device_status(reset=True)
    yield
    assert nat.device_status() == 0


@pytest.fixture(params=["sm", "tma"])
def store(request):
    """Both transports of the fused gather's peer copies."""
    from rdna2_ops.column_parallel import set_gather_store
    set_gather_store(request.param)
    yield request.param
    set_gather_store("auto")


class VirtualRanks:
    """P ranks' full outputs and gather states on one device."""

    def __init__(self, world, m, n_total, dtype):
        lib = nat.library()
        self.world, self.m, self.n = world, m, n_total
        self.outs = [torch.full((m, n_total), float("nan"), device="cuda", dtype=dtype) for _ in range(world)]
        self.states = [torch.zeros(lib.b2_gather_state_bytes(), device="cuda", dtype=torch.uint8)
                       for _ in range(world)]
        arr = ctypes.c_void_p * world
        self.out_ptrs = arr(*[t.data_ptr() for t in self.outs])
        self.state_ptrs = arr(*[t.data_ptr() for t in self.states])


def _gather_call(vr, rank, epoch, x, wq_shard, sw_shard, bias_shard, block, kind, epilogue, out_dtype, ws):
    lib = nat.library()
    m, k = x.shape
    ns = wq_shard.shape[0]
    return lib.b2_quant_linear_gather(
        kind, x.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k, k, block or 0, wq_shard.data_ptr(), k, ns,
        sw_shard.data_ptr(), sw_shard.numel(), nat.ptr(bias_shard),
        nat.DTYPE_CODE[bias_shard.dtype] if bias_shard is not None else 0, EPI[epilogue],
        nat.DTYPE_CODE[out_dtype], vr.n, rank * ns, vr.world, rank, vr.out_ptrs, vr.state_ptrs, epoch,
        ws.data_ptr(), ws.numel(), nat.stream_ptr(x.device))


def _run_all_ranks(vr, epoch, x, wq, sw, bias, block, kind, epilogue, out_dtype):
    ns = vr.n // vr.world
    lib = nat.library()
    ws = torch.empty(lib.b2_quant_linear_workspace_bytes(*x.shape), device="cuda", dtype=torch.uint8)
    for r in range(vr.world):
        s, e = r * ns, (r + 1) * ns
        swr = sw if sw.numel() == 1 else sw[s:e].contiguous()
        br = None if bias is None else bias[s:e].contiguous()
        nat.check(_gather_call(vr, r, epoch, x, wq[s:e].contiguous(), swr, br, block, kind, epilogue, out_dtype, ws),
                  "b2_quant_linear_gather")
    for r in range(vr.world):
        nat.check(lib.b2_gather_wait(vr.states[r].data_ptr(), vr.world, epoch, nat.stream_ptr(x.device)),
                  "b2_gather_wait")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("m,n_total,k,block", [(300, 1536, 512, 128), (4096, 12288, 3072, 128),
                                               (1, 512, 256, None), (513, 3072, 1024, 256)])
def test_gather_equals_single_gpu_linear(world, m, n_total, k, block, store):
    rng = np.random.default_rng(world * 7 + m)
    x = torch.from_numpy(outlier_activations(rng, m, k)).half().cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, rotation_block=block)
    bias = torch.from_numpy((rng.standard_normal(n_total) * 0.02).astype(np.float32)).half().cuda()
    ref = rdna2_ops.w8a8_linear(x, wq, sw, bias, rotation_block=block, out_dtype=torch.float16)
    vr = VirtualRanks(world, m, n_total, torch.float16)
    for epoch in (1, 2, 3):                                   # repeated calls re-use the state
        for t in vr.outs:
            t.fill_(float("nan"))
        _run_all_ranks(vr, epoch, x, wq, sw, bias, block, nat.KIND_I8, "separate", torch.float16)
        for r in range(world):
            assert torch.equal(vr.outs[r].view(torch.int16), ref.view(torch.int16)), (epoch, r)
    for st in vr.states:                                      # flags hold the last epoch, counters rearmed
        words = st.view(torch.int32).cpu().numpy()
        assert list(words[:world]) == [3] * world and words[32] == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("epilogue", ["separate", "fused", "kitchen"])
@pytest.mark.parametrize("kind", ["int8", "e4m3"])
def test_gather_dtypes_and_kinds(out_dtype, epilogue, kind, store):
    world, m, n_total, k = 4, 700, 2048, 768
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    quant = "int8" if kind == "int8" else "e4m3"
    wq, sw = qlinear.quantize_weight(w, quant=quant)
    bias = None if epilogue == "fused" else torch.from_numpy(
        (rng.standard_normal(n_total) * 0.02).astype(np.float32)).cuda()
    ref = rdna2_ops.w8a8_linear(x, wq, sw, bias, out_dtype=out_dtype, epilogue=epilogue, kind=kind)
    vr = VirtualRanks(world, m, n_total, out_dtype)
    _run_all_ranks(vr, 1, x, wq, sw, bias, None, nat.KIND_I8 if kind == "int8" else nat.KIND_E4M3, epilogue,
                   out_dtype)
    iv = torch.int32 if out_dtype == torch.float32 else torch.int16
    for r in range(world):
        assert torch.equal(vr.outs[r].view(iv), ref.view(iv)), r


def test_gather_rejects_bad_calls():
    vr = VirtualRanks(2, 64, 256, torch.float16)
    x = torch.zeros((64, 128), device="cuda", dtype=torch.float16)
    wq = torch.zeros((128, 128), device="cuda", dtype=torch.int8)
    sw = torch.ones(128, device="cuda")
    ws = torch.empty(nat.library().b2_quant_linear_workspace_bytes(64, 128), device="cuda", dtype=torch.uint8)
    lib = nat.library()
    assert _gather_call(vr, 0, 0, x, wq, sw, None, None, nat.KIND_I8, "separate", torch.float16, ws) != 0  # epoch 0
    assert _gather_call(vr, 2, 1, x, wq, sw, None, None, nat.KIND_I8, "separate", torch.float16, ws) != 0  # rank
    assert _gather_call(vr, 0, 1, x, wq[:96], sw[:96], None, None, nat.KIND_I8, "separate",
                        torch.float16, ws) != 0                                                           # N % 64
    assert lib.b2_gather_wait(vr.states[0].data_ptr() + 16, 2, 1, None) != 0                              # alignment
    torch.cuda.synchronize()


def test_gather_wait_gives_up_on_a_flag_nobody_sets():
    """A wait whose flag is never released returns after its 2 s bound with
    status 0x107; the context stays usable."""
    nat.device_status(reset=True)
    state = torch.zeros(nat.library().b2_gather_state_bytes(), device="cuda", dtype=torch.uint8)
    nat.check(nat.library().b2_gather_wait(state.data_ptr(), 2, 5, nat.stream_ptr(state.device)), "b2_gather_wait")
    assert nat.device_status(reset=True) == 0x107
    y = rdna2_ops.w8a8_linear(torch.ones((4, 128), device="cuda", dtype=torch.float16),
                              torch.ones((64, 128), device="cuda", dtype=torch.int8),
                              torch.ones(64, device="cuda"), out_dtype=torch.float32)
    assert torch.isfinite(y).all()
    assert nat.device_status() == 0


# --------------------------------------------------- copy-engine gather variant
def _gather_ce_call(vr, rank, chunks, x, wq_shard, sw_shard, bias_shard, block, kind, epilogue, out_dtype, ws):
    lib = nat.library()
    m, k = x.shape
    ns = wq_shard.shape[0]
    return lib.b2_quant_linear_gather_ce(
        kind, x.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k, k, block or 0, wq_shard.data_ptr(), k, ns,
        sw_shard.data_ptr(), sw_shard.numel(), nat.ptr(bias_shard),
        nat.DTYPE_CODE[bias_shard.dtype] if bias_shard is not None else 0, EPI[epilogue],
        nat.DTYPE_CODE[out_dtype], vr.n, rank * ns, vr.world, rank, vr.out_ptrs, vr.state_ptrs, chunks,
        ws.data_ptr(), ws.numel(), nat.stream_ptr(x.device))


def _run_all_ranks_ce(vr, chunks, x, wq, sw, bias, block, kind, epilogue, out_dtype):
    """Every rank's call first, then every rank's wait: each wait is enqueued
    after the copies and count signals it needs."""
    ns = vr.n // vr.world
    lib = nat.library()
    ws = torch.empty(lib.b2_quant_linear_workspace_bytes(*x.shape), device="cuda", dtype=torch.uint8)
    for r in range(vr.world):
        s, e = r * ns, (r + 1) * ns
        swr = sw if sw.numel() == 1 else sw[s:e].contiguous()
        br = None if bias is None else bias[s:e].contiguous()
        nat.check(_gather_ce_call(vr, r, chunks, x, wq[s:e].contiguous(), swr, br, block, kind, epilogue,
                                  out_dtype, ws), "b2_quant_linear_gather_ce")
    for r in range(vr.world):
        nat.check(lib.b2_gather_wait_ce(vr.states[r].data_ptr(), vr.world, r, nat.stream_ptr(x.device)),
                  "b2_gather_wait_ce")


@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("m,n_total,k,block", [(300, 1536, 512, 128), (4096, 12288, 3072, 128),
                                               (1, 512, 256, None), (1100, 3072, 1024, 256)])
def test_gather_ce_equals_single_gpu_linear(chunks, world, m, n_total, k, block):
    """Chunked GEMM + copy-engine transfer: every rank's full output equals
    the single-GPU linear bit for bit over three calls; each rank's state
    ends with every peer's count and its own sequence number at 3."""
    rng = np.random.default_rng(world * 5 + m + chunks)
    x = torch.from_numpy(outlier_activations(rng, m, k)).half().cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, rotation_block=block)
    bias = torch.from_numpy((rng.standard_normal(n_total) * 0.02).astype(np.float32)).half().cuda()
    ref = rdna2_ops.w8a8_linear(x, wq, sw, bias, rotation_block=block, out_dtype=torch.float16)
    vr = VirtualRanks(world, m, n_total, torch.float16)
    for call in (1, 2, 3):
        for t in vr.outs:
            t.fill_(float("nan"))
        _run_all_ranks_ce(vr, chunks, x, wq, sw, bias, block, nat.KIND_I8, "separate", torch.float16)
        for r in range(world):
            assert torch.equal(vr.outs[r].view(torch.int16), ref.view(torch.int16)), (call, r)
    for r, st in enumerate(vr.states):
        words = st.view(torch.int32).cpu().numpy()
        counts = words[8:8 + world]
        assert all(counts[q] == (0 if q == r else 3) for q in range(world)) and words[40] == 3, (r, words[:48])
    assert nat.device_status() == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("kind", ["int8", "e4m3"])
def test_gather_ce_dtypes_and_kinds(out_dtype, kind):
    world, m, n_total, k = 4, 700, 2048, 768
    rng = np.random.default_rng(13)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, quant="int8" if kind == "int8" else "e4m3")
    bias = torch.from_numpy((rng.standard_normal(n_total) * 0.02).astype(np.float32)).cuda()
    ref = rdna2_ops.w8a8_linear(x, wq, sw, bias, out_dtype=out_dtype, epilogue="kitchen", kind=kind)
    vr = VirtualRanks(world, m, n_total, out_dtype)
    _run_all_ranks_ce(vr, 2, x, wq, sw, bias, None, nat.KIND_I8 if kind == "int8" else nat.KIND_E4M3, "kitchen",
                      out_dtype)
    iv = torch.int32 if out_dtype == torch.float32 else torch.int16
    for r in range(world):
        assert torch.equal(vr.outs[r].view(iv), ref.view(iv)), r


def test_gather_ce_graph_replay():
    """A captured step (every rank's call and wait) replays with fresh inputs:
    the wait advances its own sequence number, so no host value is baked in."""
    world, m, n_total, k = 2, 1024, 2048, 1024
    rng = np.random.default_rng(17)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).half().cuda()
    w = torch.from_numpy((rng.standard_normal((n_total, k)) * 0.02).astype(np.float32)).cuda()
    wq, sw = qlinear.quantize_weight(w, rotation_block=128)
    vr = VirtualRanks(world, m, n_total, torch.float16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _run_all_ranks_ce(vr, 2, x, wq, sw, None, 128, nat.KIND_I8, "separate", torch.float16)  # warm-up: streams
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _run_all_ranks_ce(vr, 2, x, wq, sw, None, 128, nat.KIND_I8, "separate", torch.float16)
    for step in range(3):
        x.copy_(torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).half())
        for t in vr.outs:
            t.fill_(float("nan"))
        graph.replay()
        ref = rdna2_ops.w8a8_linear(x, wq, sw, None, rotation_block=128, out_dtype=torch.float16)
        for r in range(world):
            assert torch.equal(vr.outs[r].view(torch.int16), ref.view(torch.int16)), (step, r)
    torch.cuda.synchronize()
    words = vr.states[0].view(torch.int32).cpu().numpy()
    assert words[9] == 4 and words[40] == 4
    del graph
    assert nat.device_status() == 0


def test_gather_ce_rejects_bad_calls_and_wait_gives_up():
    vr = VirtualRanks(2, 64, 256, torch.float16)
    x = torch.zeros((64, 128), device="cuda", dtype=torch.float16)
    wq = torch.zeros((128, 128), device="cuda", dtype=torch.int8)
    sw = torch.ones(128, device="cuda")
    ws = torch.empty(nat.library().b2_quant_linear_workspace_bytes(64, 128), device="cuda", dtype=torch.uint8)
    lib = nat.library()
    assert _gather_ce_call(vr, 0, 0, x, wq, sw, None, None, nat.KIND_I8, "separate", torch.float16, ws) != 0
    assert _gather_ce_call(vr, 0, 9, x, wq, sw, None, None, nat.KIND_I8, "separate", torch.float16, ws) != 0
    assert _gather_ce_call(vr, 2, 1, x, wq, sw, None, None, nat.KIND_I8, "separate", torch.float16, ws) != 0
    assert lib.b2_gather_wait_ce(vr.states[0].data_ptr() + 16, 2, 0, None) != 0
    torch.cuda.synchronize()
    nat.device_status(reset=True)
    state = torch.zeros(lib.b2_gather_state_bytes(), device="cuda", dtype=torch.uint8)
    nat.check(lib.b2_gather_wait_ce(state.data_ptr(), 2, 0, nat.stream_ptr(state.device)), "b2_gather_wait_ce")
    assert nat.device_status(reset=True) == 0x107
    assert torch.isfinite(rdna2_ops.w8a8_linear(x + 1, wq + 1, sw, out_dtype=torch.float32)).all()
    assert nat.device_status() == 0
