"""Column-parallel sharding and output reassembly.

CPU: world_size-2 gloo process groups with the CPU oracle as the rank-local
linear -- the gathered output must equal the unsharded oracle linear bit for
bit, and a rank that dies must surface as an error on its peer (short
process-group timeout), not a hang.
GPU (2+ devices): NCCL ranks running the B200 kernels, bit-identical to the
single-GPU linear."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from rdna2_ops.column_parallel import ColumnParallelLinear, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_covers_and_aligns():
    for n, world, align in ((12288, 8, 128), (100, 3, 1), (3072, 2, 16), (5, 4, 1)):
        spans = [shard_range(n, world, r, align) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c
        for s, e in spans[:-1]:
            if e > s:
                assert (e - s) % align == 0
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _oracle_local(x, w, sw, b):
    xq, sx = oracle.act_quant_int8(x.numpy(), oracle.F32, 128)
    acc = oracle.gemm_s8(xq, w.numpy())
    return torch.from_numpy(oracle.epilogue_s32(acc, sx, sw.numpy(), b.numpy(), oracle.F32))


def _gloo_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        rng = np.random.default_rng(5)
        m, n, k = 12, 64, 256
        x = torch.from_numpy(rng.standard_normal((2, m // 2, k)).astype(np.float32))
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, 128))
        bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
        layer = ColumnParallelLinear.from_full(torch.from_numpy(wq), torch.from_numpy(sw),
                                               torch.from_numpy(bias), local_fn=_oracle_local)
        y = layer(x)
        ref = _oracle_local(x.reshape(-1, k), torch.from_numpy(wq), torch.from_numpy(sw),
                            torch.from_numpy(bias)).reshape(2, m // 2, n)
        q.put((rank, bool(torch.equal(y.view(torch.int32), ref.view(torch.int32))), tuple(y.shape)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_match_unsharded_oracle():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok, _ in res) and res[0][2] == (2, 6, 64)


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)                       # leaves between steps, before the collective
    try:
        t = torch.zeros(4)
        dist.all_gather_into_tensor(torch.zeros(8), t)
        q.put("completed")
    except Exception as exc:              # the peer's absence surfaces as an error
        q.put("error:" + type(exc).__name__)


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert q.get(timeout=10).startswith("error:")


def _nccl_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from rdna2_ops import qlinear, w8a8_linear
        g = torch.Generator(device="cuda").manual_seed(20261106)
        m, n, k = 1024, 3072 * 2, 3072
        x = torch.randn((m, k), generator=g, device="cuda").half()
        w = torch.randn((n, k), generator=g, device="cuda") * 0.02
        wq, sw = qlinear.quantize_weight(w, rotation_block=128)
        bias = (torch.randn(n, generator=g, device="cuda") * 0.02).half()
        layer = ColumnParallelLinear.from_full(wq, sw, bias, rotation_block=128,
                                               out_dtype=torch.float16)
        y = layer(x)
        ref = w8a8_linear(x, wq, sw, bias, rotation_block=128, out_dtype=torch.float16)
        q.put((rank, bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_column_parallel_bit_identical():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert all(ok for _, ok in sorted(q.get(timeout=10) for _ in range(2)))


def _peer_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    g = None
    try:
        from rdna2_ops import qlinear, w8a8_linear
        from rdna2_ops.column_parallel import ColumnParallelStack, PeerGather
        gen = torch.Generator(device="cuda").manual_seed(20261106)
        m, n, k = 1000, 768 * world, 3072
        x = torch.randn((m, k), generator=gen, device="cuda").half()
        w = torch.randn((n, k), generator=gen, device="cuda") * 0.02
        wq, sw = qlinear.quantize_weight(w, rotation_block=128)
        bias = (torch.randn(n, generator=gen, device="cuda") * 0.02).half()
        g = PeerGather(8192 * 2048, torch.float16)
        ref = w8a8_linear(x, wq, sw, bias, rotation_block=128, out_dtype=torch.float16)
        ok = True
        from rdna2_ops.column_parallel import set_gather_store
        for mode, store in (("peer", "sm"), ("ce", "auto"), ("peer", "tma"), ("ce", "auto"), ("peer", "auto")):
            set_gather_store(store)                 # every variant, interleaved on the same buffers
            layer = ColumnParallelLinear.from_full(wq, sw, bias, rotation_block=128, out_dtype=torch.float16,
                                                   gather=mode, peers=g)
            for _ in range(5):                      # both ring buffers, several calls
                y = layer(x)
                ok &= bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
        # two DiT blocks (hidden 512), column-parallel with the peer gather,
        # against the same chain of single-GPU fused linears
        hid, blocks = 512, []
        for _ in range(2):
            blk = []
            for nn_, kk in ((3 * hid, hid), (hid, hid), (4 * hid, hid), (hid, 4 * hid)):
                wf = torch.randn((nn_, kk), generator=gen, device="cuda") / kk ** 0.5
                blk.append(qlinear.quantize_weight(wf, rotation_block=128))
            blocks.append(blk)
        x0 = torch.randn((256, hid), generator=gen, device="cuda").half()
        yr = x0
        for blk in blocks:
            (q1, s1), (q2, s2), (q3, s3), (q4, s4) = blk
            qkv = w8a8_linear(yr, q1, s1, rotation_block=128, out_dtype=torch.float16)
            o = w8a8_linear(qkv[:, :hid], q2, s2, rotation_block=128, out_dtype=torch.float16)
            yr = w8a8_linear(w8a8_linear(o, q3, s3, rotation_block=128, out_dtype=torch.float16), q4, s4,
                             rotation_block=128, out_dtype=torch.float16)
        ok_stack = True
        for mode, store in (("peer", "sm"), ("peer", "tma"), ("ce", "auto")):
            set_gather_store(store)
            stack = ColumnParallelStack(blocks, peers=g, gather=mode)
            ys = stack(x0)
            ok_stack &= bool(torch.equal(ys.view(torch.int16), yr.view(torch.int16)))
        # the same chain with INT8 activations exchanged between the layers
        # (hidden 128 * world: every shard width a multiple of the block)
        from rdna2_ops.column_parallel import ActivationExchange
        hid8, blocks8 = 128 * world, []
        for _ in range(2):
            blk = []
            for nn_, kk in ((3 * hid8, hid8), (hid8, hid8), (4 * hid8, hid8), (hid8, 4 * hid8)):
                wf = torch.randn((nn_, kk), generator=gen, device="cuda") / kk ** 0.5
                blk.append(qlinear.quantize_weight(wf, rotation_block=128))
            blocks8.append(blk)
        x8 = torch.randn((300, hid8), generator=gen, device="cuda").half()
        yr8 = x8
        for blk in blocks8:
            (q1, s1), (q2, s2), (q3, s3), (q4, s4) = blk
            qkv = w8a8_linear(yr8, q1, s1, rotation_block=128, out_dtype=torch.float16)
            o = w8a8_linear(qkv[:, :hid8], q2, s2, rotation_block=128, out_dtype=torch.float16)
            yr8 = w8a8_linear(w8a8_linear(o, q3, s3, rotation_block=128, out_dtype=torch.float16), q4, s4,
                              rotation_block=128, out_dtype=torch.float16)
        for fused in (True, False):                 # one-launch and two-launch exchanges
            ex = ActivationExchange(300, 4 * hid8, fused=fused)
            try:
                stack8 = ColumnParallelStack(blocks8, peers=g, activations="int8", codes=ex)
                for _ in range(3):                  # buffers and epochs reused across calls
                    y8 = stack8(x8)
                    ok_stack &= bool(torch.equal(y8.view(torch.int16), yr8.view(torch.int16)))
            finally:
                ex.close()
        from rdna2_ops import _native as nat
        q.put((rank, ok, ok_stack, nat.device_status()))
    finally:
        if g is not None:
            g.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_gather_column_parallel_bit_identical():
    """Every rank's reassembled output (the gather inside the GEMM epilogue,
    or by copy engines behind a chunked GEMM, over NVLink) equals the
    single-GPU fused linear bit for bit, over several calls; a 2-block
    column-parallel DiT stack equals the 1-GPU stack with either gather and
    with INT8 activations exchanged between the layers."""
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(ok and ok_stack and st == 0 for _, ok, ok_stack, st in res), res


def test_shard_overlap_ranges():
    from rdna2_ops.column_parallel import shard_overlap
    assert shard_overlap(0, 768, 0, 512) == (0, 512)
    assert shard_overlap(768, 768, 0, 512) == (512, 512)         # past the range: empty, at its end
    assert shard_overlap(0, 512, 512, 2048) == (512, 512)        # before the range: empty, at its start
    assert shard_overlap(2304, 1152, 0, 3072) == (2304, 3072)
    assert shard_overlap(1024, 512, 512, 2048) == (1024, 1536)
