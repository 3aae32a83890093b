"""Column-parallel (N-sharded) quantized linear across the GPUs of one node.

Each rank owns the weight rows [start, stop) of the output dimension N
(plus their per-channel scales and bias), receives the replicated
activations and runs the fused linear locally (rotation + per-token
quantization + tcgen05 GEMM + epilogue).  Per-token scales depend only on
the activation row, which every rank sees whole, so the reassembled output
is bit-identical to the single-GPU linear.

Reassembly of the full Y[M, N] on every rank, two ways:

* ``gather="peer"`` (default where it applies): the GEMM epilogue itself
  writes every output tile into the same columns of every rank's full output
  buffer over NVLink (C ABI b2_quant_linear_gather), so the transfer overlaps
  the multiplication tile by tile and Y arrives row-major with no permute
  pass.  Buffers come from a PeerGather, which maps every rank's buffers into
  every process once (CUDA IPC) and rotates through two of them.
* ``gather="ce"``: the same buffers, the linear in M-chunks, and each
  chunk's block carried to every peer by the copy engines while the next
  chunk is multiplied (C ABI b2_quant_linear_gather_ce + b2_gather_wait_ce);
  counter-based completion, so a step can be captured in a CUDA graph.
* ``gather="nccl"``: the local linear, then one NCCL all_gather_into_tensor
  into [P, M, N/P] and a permute to [M, N] (any shard width, any local_fn).

The reference is single-GPU (no collectives anywhere); this module is the
multi-GPU execution the north star asks for, with torch.distributed as the
plumbing (one process per GPU, NCCL backend).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as nat
from .qlinear import EPILOGUES, _block, _operand, _rows_2d, w8a8_linear


def shard_range(n, world, rank, align=1):
    """Contiguous [start, stop) of `n` columns owned by `rank`; every shard but
    possibly the last is a multiple of `align` and all shards are equal when
    n is divisible by world * align."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    units = -(-n // align)
    per = -(-units // world)
    start = min(n, rank * per * align)
    stop = min(n, (rank + 1) * per * align)
    return start, stop


def set_gather_store(mode):
    """Transport of the fused gather's peer copies, process-wide: "auto",
    "sm" (16-byte stores from the epilogue warps) or "tma" (TMA stores
    through per-peer tensor maps).  Outputs are identical for every choice."""
    codes = {"auto": 0, "sm": 1, "tma": 2}
    if mode not in codes:
        raise ValueError("gather store must be 'auto', 'sm' or 'tma'")
    nat.check(nat.library().b2_set_gather_store(codes[mode]), "b2_set_gather_store")


def ce_chunks(world):
    """M-chunks of the copy-engine gather: enough to overlap the transfer
    with the GEMM while each rank's share of the GEMM is still large (4 at 2
    ranks, 2 at 3-4); one chunk beyond, where the transfer dwarfs the GEMM."""
    return 1 if world == 1 else 4 if world == 2 else 2 if world <= 4 else 1


class PeerGather:
    """Output buffers shared by the ranks of a process group for the fused
    column-parallel gather.

    Every rank allocates `buffers` flat output buffers of `capacity` elements
    of `dtype` and one gather-state block; the IPC handles are exchanged once
    (all_gather_object over `group`) and each rank maps every peer's buffers.
    Calls rotate through the buffers, one epoch per call, in the same order on
    every rank.  The result of a call lives in the rank's own buffer until
    the call `buffers` calls later overwrites it: read it on the calling
    stream before issuing the next gathered call (a consumer on another
    stream must be waited on by the calling stream first).

    `exchange(obj) -> list` (one entry per rank) replaces all_gather_object
    for tests."""

    def __init__(self, capacity, dtype, *, group=None, buffers=2, device=None, exchange=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.capacity = int(capacity)
        self.lib = nat.library()
        self.local = [torch.empty(self.capacity, device=self.device, dtype=dtype) for _ in range(buffers)]
        self.state = torch.zeros(self.lib.b2_gather_state_bytes(), device=self.device, dtype=torch.uint8)
        if self.state.data_ptr() % 256:
            raise RuntimeError("gather state must be 256-byte aligned")
        self.epoch = 0
        self._imported = []
        mine = [self._export(t) for t in self.local + [self.state]]
        if exchange is not None:
            everyone = exchange(mine)
        elif self.world == 1:
            everyone = [mine]
        else:
            everyone = [None] * self.world
            dist.all_gather_object(everyone, mine, group=group)
        ptrs = [[None] * self.world for _ in range(buffers + 1)]
        for r, entries in enumerate(everyone):
            for i, (handle, offset) in enumerate(entries):
                ptrs[i][r] = (self.local + [self.state])[i].data_ptr() if r == self.rank \
                    else self._import(handle, offset)
        arr = ctypes.c_void_p * self.world
        self.outs = [arr(*p) for p in ptrs[:buffers]]
        self.states = arr(*ptrs[buffers])
        torch.cuda.synchronize(self.device)

    def _export(self, t):
        h = ctypes.create_string_buffer(self.lib.b2_ipc_handle_bytes())
        off = ctypes.c_uint64(0)
        nat.check(self.lib.b2_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "b2_ipc_export")
        return bytes(h.raw), int(off.value)

    def _import(self, handle, offset):
        ptr = ctypes.c_void_p()
        nat.check(self.lib.b2_ipc_import(handle, offset, ctypes.byref(ptr)), "b2_ipc_import")
        self._imported.append(handle)
        return ptr.value

    def close(self, barrier=True):
        """Unmap the peers' buffers.  Collective by default: every rank calls
        it after its last gathered call, and it returns only when every rank
        has unmapped, so no rank frees buffers a peer still maps (a caller
        that synchronizes the ranks itself passes barrier=False)."""
        torch.cuda.synchronize(self.device)
        while self._imported:
            nat.check(self.lib.b2_ipc_release(self._imported.pop()), "b2_ipc_release")
        if barrier and self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)

    def next_slot(self):
        """(epoch, buffer index) of the next call."""
        self.epoch += 1
        return self.epoch, self.epoch % len(self.local)

    def wait(self, epoch, stream):
        nat.check(self.lib.b2_gather_wait(self.state.data_ptr(), self.world, epoch, stream), "b2_gather_wait")


class ColumnParallelLinear:
    """y = x @ W.T (+ bias), W sharded along N over `group`.

    local_fn(x2d, w_shard, w_scale_shard, bias_shard) -> y_shard computes the
    rank's columns for the "nccl" reassembly; the default is the B200 fused
    linear (w8a8_linear with the given rotation / epilogue / kind).  The
    "peer" reassembly runs the fused linear with the gather in its epilogue
    and needs a PeerGather (`peers`) sized for M x N outputs of out_dtype.
    """

    def __init__(self, w_shard, w_scale_shard, bias_shard, n_total, *, group=None,
                 rotation_block=None, out_dtype=None, epilogue="separate", kind="int8",
                 local_fn=None, gather="auto", peers=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_total = n_total
        if n_total % self.world:
            raise ValueError("N must divide evenly across ranks for the all-gather")
        self.n_shard = n_total // self.world
        if w_shard.shape[0] != self.n_shard:
            raise ValueError("weight shard does not match N / world")
        if gather not in ("auto", "peer", "ce", "nccl"):
            raise ValueError("gather must be 'auto', 'peer', 'ce' or 'nccl'")
        self.w, self.sw, self.bias = w_shard, w_scale_shard, bias_shard
        self.kw = dict(rotation_block=rotation_block, out_dtype=out_dtype, epilogue=epilogue, kind=kind)
        self.local_fn = local_fn or (lambda x, w, sw, b: w8a8_linear(x, w, sw, b, **self.kw))
        peer_ok = local_fn is None and self.n_shard % 64 == 0 and kind in ("int8", "e4m3")
        if gather in ("peer", "ce") and not peer_ok:
            raise ValueError("the peer and copy-engine gathers need the built-in linear and N / world % 64 == 0")
        if gather == "auto":
            gather = "peer" if (peer_ok and peers is not None) else "nccl"
        self.gather_mode = gather
        self.peers = peers
        self._workspace = None

    @classmethod
    def from_full(cls, w_q, w_scale, bias=None, *, group=None, **kw):
        """Slice this rank's shard out of full [N,K] weight tensors."""
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        n = w_q.shape[0]
        s, e = shard_range(n, world, rank)
        sw = w_scale if w_scale.numel() == 1 else w_scale[s:e].contiguous()
        b = None if bias is None else bias[s:e].contiguous()
        return cls(w_q[s:e].contiguous(), sw, b, n, group=group, **kw)

    def forward_local(self, x):
        """This rank's output columns [..., N / world]."""
        x2 = x.reshape(-1, x.shape[-1])
        y = self.local_fn(x2, self.w, self.sw, self.bias)
        return y.reshape(*x.shape[:-1], y.shape[-1])

    def _forward_peer(self, x):
        """Fused linear whose epilogue writes every rank's copy of Y."""
        g = self.peers
        out_dtype = self.kw["out_dtype"] or x.dtype
        if g is None or g.dtype != out_dtype:
            raise ValueError("the peer gather needs a PeerGather of the output dtype")
        dev = nat.require_device(x, self.w, self.sw, self.bias)
        nat.eager_only(x, self.bias)
        x2 = _rows_2d(x)
        m, k = x2.shape
        if m * self.n_total > g.capacity:
            raise ValueError(f"PeerGather holds {g.capacity} outputs, this call needs {m * self.n_total}")
        epoch, slot = g.next_slot()
        y = g.local[slot][: m * self.n_total].view(m, self.n_total)
        if m == 0:
            return y.reshape(*x.shape[:-1], self.n_total)
        lib = nat.library()
        need = lib.b2_quant_linear_workspace_bytes(m, k)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty(need, device=dev, dtype=torch.uint8)
        w_t, ldw = _operand(self.w.view(torch.uint8), 1) or (None, None)
        if w_t is None:
            raise ValueError("weight shard rows must be 16-byte aligned")
        kind = nat.KIND_I8 if self.kw["kind"] == "int8" else nat.KIND_E4M3
        stream = nat.stream_ptr(dev)
        common = (kind, x2.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k, x2.stride(0) if m > 1 else k,
                  _block(self.kw["rotation_block"], k), w_t.data_ptr(), ldw, self.n_shard, self.sw.data_ptr(),
                  self.sw.numel(), nat.ptr(self.bias), nat.DTYPE_CODE[self.bias.dtype] if self.bias is not None else 0,
                  EPILOGUES[self.kw["epilogue"]], nat.DTYPE_CODE[out_dtype], self.n_total, self.rank * self.n_shard,
                  self.world, self.rank, g.outs[slot], g.states)
        if self.gather_mode == "ce":
            nat.check(lib.b2_quant_linear_gather_ce(*common, ce_chunks(self.world), self._workspace.data_ptr(),
                                                    self._workspace.numel(), stream), "b2_quant_linear_gather_ce")
            nat.check(lib.b2_gather_wait_ce(g.state.data_ptr(), self.world, self.rank, stream), "b2_gather_wait_ce")
        else:
            nat.check(lib.b2_quant_linear_gather(*common, epoch, self._workspace.data_ptr(), self._workspace.numel(),
                                                 stream), "b2_quant_linear_gather")
            g.wait(epoch, stream)
        return y.reshape(*x.shape[:-1], self.n_total)

    def forward(self, x, gather=True):
        if gather and self.gather_mode in ("peer", "ce"):
            return self._forward_peer(x)
        y = self.forward_local(x)
        if not gather or self.world == 1:
            return y
        lead = y.shape[:-1]
        shard = y.reshape(-1, y.shape[-1]).contiguous()
        m, ns = shard.shape
        buf = torch.empty((self.world * m, ns), device=shard.device, dtype=shard.dtype)
        dist.all_gather_into_tensor(buf, shard, group=self.group)
        full = buf.view(self.world, m, ns).permute(1, 0, 2).reshape(m, self.world * ns)
        return full.reshape(*lead, self.world * ns)

    __call__ = forward


class ColumnParallelStack:
    """The linear chain of BASELINE config 5's DiT blocks, column-parallel:
    per block QKV [3h, h], the out projection on the Q third of the QKV
    output (read in place through its row stride), up [4h, h] and down
    [h, 4h], every one a W8A8 fused linear with block rotation whose output is
    reassembled on every rank before the next linear reads it.  (Attention is
    not on this path.)  `blocks` holds, per block, four (w_q [N,K], w_scale)
    pairs of the full quantized weights; each rank keeps only its shards.
    With a PeerGather the gathers run inside the GEMM epilogues and the layer
    outputs alternate between its two buffers."""

    def __init__(self, blocks, *, group=None, rotation_block=128, out_dtype=torch.float16, peers=None,
                 gather="auto"):
        self.hidden = blocks[0][1][0].shape[0]
        self.layers = [[ColumnParallelLinear.from_full(wq, sw, None, group=group, rotation_block=rotation_block,
                                                       out_dtype=out_dtype, peers=peers, gather=gather)
                        for wq, sw in blk] for blk in blocks]

    def forward(self, x):
        h = self.hidden
        for qkv_l, out_l, up_l, down_l in self.layers:
            qkv = qkv_l(x)
            o = out_l(qkv[:, :h])
            x = down_l(up_l(o))
        return x

    __call__ = forward
