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


def _map_peers(lib, tensors, world, rank, group, exchange):
    """Export every tensor's IPC handle, exchange the handles (one
    all_gather_object, or `exchange` in tests) and map every peer's tensors.
    Returns (per tensor, a ctypes array of the world ranks' device pointers
    -- this rank's own tensor at index `rank`) and the imported handles."""
    def export(t):
        h = ctypes.create_string_buffer(lib.b2_ipc_handle_bytes())
        off = ctypes.c_uint64(0)
        nat.check(lib.b2_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "b2_ipc_export")
        return bytes(h.raw), int(off.value)

    mine = [export(t) for t in tensors]
    if exchange is not None:
        everyone = exchange(mine)
    elif world == 1:
        everyone = [mine]
    else:
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
    imported = []
    ptrs = [[None] * world for _ in tensors]
    for r, entries in enumerate(everyone):
        for i, (handle, offset) in enumerate(entries):
            if r == rank:
                ptrs[i][r] = tensors[i].data_ptr()
                continue
            ptr = ctypes.c_void_p()
            nat.check(lib.b2_ipc_import(handle, offset, ctypes.byref(ptr)), "b2_ipc_import")
            imported.append(handle)
            ptrs[i][r] = ptr.value
    arr = ctypes.c_void_p * world
    return [arr(*p) for p in ptrs], imported


def _unmap_peers(lib, imported):
    while imported:
        nat.check(lib.b2_ipc_release(imported.pop()), "b2_ipc_release")


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
        arrays, self._imported = _map_peers(self.lib, self.local + [self.state], self.world, self.rank, group,
                                            exchange)
        self.outs = arrays[:buffers]
        self.states = arrays[buffers]
        torch.cuda.synchronize(self.device)

    def close(self, barrier=True):
        """Unmap the peers' buffers.  Collective by default: every rank calls
        it after its last gathered call, and it returns only when every rank
        has unmapped, so no rank frees buffers a peer still maps (a caller
        that synchronizes the ranks itself passes barrier=False)."""
        torch.cuda.synchronize(self.device)
        _unmap_peers(self.lib, self._imported)
        if barrier and self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)

    def next_slot(self):
        """(epoch, buffer index) of the next call."""
        self.epoch += 1
        return self.epoch, self.epoch % len(self.local)

    def wait(self, epoch, stream):
        nat.check(self.lib.b2_gather_wait(self.state.data_ptr(), self.world, epoch, stream), "b2_gather_wait")


class ActivationExchange:
    """Buffers of the column-parallel INT8 activation exchange (C ABI
    b2_shard_amax / b2_shard_codes): per rank a per-row absmax exchange
    buffer [world, m_max] fp32, two alternating code buffers [m_max,
    round16(k_max)] int8 that the peers write into, the row scales [m_max]
    (local) and one completion state per phase, all mapped by every peer
    like PeerGather's buffers.  `close()` is collective like
    PeerGather.close.  fused=True runs both phases of an exchange in one
    cooperative kernel (b2_shard_exchange; one rank per GPU), False as two
    kernels with a wait between them."""

    def __init__(self, m_max, k_max, *, group=None, device=None, exchange=None, fused=True):
        self.group = group
        self.fused = bool(fused)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.lib = nat.library()
        self.m_max = int(m_max)
        self.ldq = -(-int(k_max) // 16) * 16
        sb = self.lib.b2_gather_state_bytes()
        self.xchg = torch.zeros(self.world * self.m_max, device=self.device, dtype=torch.float32)
        self.codes = [torch.empty((self.m_max, self.ldq), device=self.device, dtype=torch.int8) for _ in range(2)]
        self.scale = torch.empty(self.m_max, device=self.device, dtype=torch.float32)
        self.state_amax = torch.zeros(sb, device=self.device, dtype=torch.uint8)
        self.state_codes = torch.zeros(sb, device=self.device, dtype=torch.uint8)
        for st in (self.state_amax, self.state_codes):
            if st.data_ptr() % 256:
                raise RuntimeError("exchange state must be 256-byte aligned")
        arrays, self._imported = _map_peers(
            self.lib, [self.xchg] + self.codes + [self.state_amax, self.state_codes], self.world, self.rank, group,
            exchange)
        self.xchg_ptrs = arrays[0]
        self.code_ptrs = arrays[1:3]
        self.amax_states, self.code_states = arrays[3], arrays[4]
        self.epoch_amax = 0
        self.epoch_codes = 0
        torch.cuda.synchronize(self.device)

    def close(self, barrier=True):
        torch.cuda.synchronize(self.device)
        _unmap_peers(self.lib, self._imported)
        if barrier and self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)

    def exchange_slice(self, y, m, width, ldy, block, dst, col0, stream):
        """Every rank's codes and this rank's scales for the next layer from
        this rank's slice y [m, width] (row stride ldy) of the layer output:
        the two phases and their waits, enqueued on `stream`.  `dst` selects
        the code buffer, `col0` the slice's first column in the next layer's
        input."""
        lib = self.lib
        ptr = y if isinstance(y, int) else y.data_ptr()
        self.epoch_amax += 1
        self.epoch_codes += 1
        if self.fused:                         # both phases in one cooperative launch
            nat.check(lib.b2_shard_exchange(ptr, nat.F16, m, width, ldy, block, 0, self.world, self.rank,
                                            self.xchg_ptrs, self.amax_states, self.epoch_amax, self.code_ptrs[dst],
                                            self.ldq, col0, self.scale.data_ptr(), self.code_states,
                                            self.epoch_codes, stream), "b2_shard_exchange")
        else:
            nat.check(lib.b2_shard_amax(ptr, nat.F16, m, width, ldy, block, self.world, self.rank,
                                        self.xchg_ptrs, self.amax_states, self.epoch_amax, stream), "b2_shard_amax")
            nat.check(lib.b2_gather_wait(self.state_amax.data_ptr(), self.world, self.epoch_amax, stream),
                      "b2_gather_wait")
            nat.check(lib.b2_shard_codes(ptr, nat.F16, m, width, ldy, block, 0, self.world, self.rank,
                                         self.xchg.data_ptr(), self.code_ptrs[dst], self.ldq, col0,
                                         self.scale.data_ptr(), self.code_states, self.epoch_codes, stream),
                      "b2_shard_codes")
        nat.check(lib.b2_gather_wait(self.state_codes.data_ptr(), self.world, self.epoch_codes, stream),
                  "b2_gather_wait")


def shard_overlap(c0, width, lo, hi):
    """This rank's part [a, b) of the next layer's input columns [lo, hi),
    given its output columns [c0, c0 + width); (a, a) when they miss."""
    a, b = max(c0, lo), min(c0 + width, hi)
    return (a, b) if a < b else (max(lo, min(c0, hi)), max(lo, min(c0, hi)))


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
    [h, 4h], every one a W8A8 fused linear with block rotation.  (Attention
    is not on this path.)  `blocks` holds, per block, four (w_q [N,K],
    w_scale) pairs of the full quantized weights; each rank keeps only its
    shards.

    activations="fp16": every layer output is reassembled on every rank
    before the next linear reads it (with a PeerGather the gathers run
    inside the GEMM epilogues).  activations="int8" (needs `codes`, an
    ActivationExchange, and `peers`): only the next layer's input travels,
    as INT8 codes -- each rank rotates and reduces its own slice of the
    layer output, the per-row absmax slices are exchanged and each rank
    quantizes its slice with the row's global scale into every rank's code
    buffer; the first layer quantizes the replicated input locally and the
    last layer's fp16 output is gathered by the fused GEMM epilogue (on one
    rank it is the plain fused chain).  Both modes are bit-identical to the
    same chain of single-GPU fused linears.
    Every rank's shard widths must be multiples of the rotation block (and
    of 64) in int8 mode."""

    def __init__(self, blocks, *, group=None, rotation_block=128, out_dtype=torch.float16, peers=None,
                 gather="auto", activations="fp16", codes=None):
        if activations not in ("fp16", "int8"):
            raise ValueError("activations must be 'fp16' or 'int8'")
        self.hidden = blocks[0][1][0].shape[0]
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if activations == "int8" and world == 1:
            activations = "fp16"               # one rank: nothing to exchange, the plain fused chain
        self.activations = activations
        if activations == "fp16":
            self.layers = [[ColumnParallelLinear.from_full(wq, sw, None, group=group,
                                                           rotation_block=rotation_block, out_dtype=out_dtype,
                                                           peers=peers, gather=gather)
                            for wq, sw in blk] for blk in blocks]
            return
        if codes is None or peers is None:
            raise ValueError("activations='int8' needs codes=ActivationExchange and peers=PeerGather")
        if out_dtype != torch.float16:
            raise ValueError("activations='int8' exchanges fp16 layer outputs")
        self.codes, self.peers = codes, peers
        self.world, self.rank = codes.world, codes.rank
        self.block = rotation_block
        h = self.hidden
        self.chain = []                        # (w shard, w_scale shard, K, N shard, col0, next-input range)
        flat = [(wq, sw) for blk in blocks for wq, sw in blk]
        nxt = [(0, h), (0, h), (0, 4 * h), (0, h)]
        for i, (wq, sw) in enumerate(flat):
            n, k = wq.shape
            if n % self.world:
                raise ValueError("N must divide by the world size")
            ns = n // self.world
            c0 = self.rank * ns
            if ns % 64 or (self.block and self.block > 1 and ns % self.block):
                raise ValueError("int8 activations need shard widths that are multiples of the rotation block")
            if k > codes.ldq:
                raise ValueError("ActivationExchange k_max is smaller than a layer's K")
            rng = None if i == len(flat) - 1 else nxt[i % 4]
            self.chain.append((wq[c0:c0 + ns].contiguous(), sw[c0:c0 + ns].contiguous(), k, ns, c0, rng))
        self._ys = {}

    def _y(self, m, ns, device):
        key = (m, ns)
        if key not in self._ys:
            self._ys[key] = torch.empty((m, ns), device=device, dtype=torch.float16)
        return self._ys[key]

    def _forward_int8(self, x):
        lib, ex, g = nat.library(), self.codes, self.peers
        dev = x.device
        stream = nat.stream_ptr(dev)
        x2 = _rows_2d(x)
        m, k0 = x2.shape
        if m > ex.m_max:
            raise ValueError("more rows than the ActivationExchange holds")
        if m * self.chain[-1][3] * self.world > g.capacity:
            raise ValueError("output larger than the PeerGather buffers")
        block = _block(self.block, k0)
        cur = 0
        nat.check(lib.b2_act_quant(x2.data_ptr(), nat.DTYPE_CODE[x.dtype], m, k0, x2.stride(0) if m > 1 else k0,
                                   block, 0, ex.codes[cur].data_ptr(), ex.ldq, ex.scale.data_ptr(), stream),
                  "b2_act_quant")
        for w, sw, k, ns, c0, rng in self.chain:
            if rng is None:                    # last layer: fp16 output gathered in the epilogue
                n_total = ns * self.world
                epoch, slot = g.next_slot()
                nat.check(lib.b2_qgemm_gather(nat.KIND_I8, ex.codes[cur].data_ptr(), ex.ldq, ex.scale.data_ptr(),
                                              w.data_ptr(), k, m, ns, k, sw.data_ptr(), ns, None, 0,
                                              EPILOGUES["separate"], nat.F16, n_total, c0, self.world, self.rank,
                                              g.outs[slot], g.states, epoch, stream), "b2_qgemm_gather")
                g.wait(epoch, stream)
                return g.local[slot][: m * n_total].view(m, n_total).reshape(*x.shape[:-1], n_total)
            y = self._y(m, ns, dev)
            nat.check(lib.b2_qgemm(nat.KIND_I8, ex.codes[cur].data_ptr(), ex.ldq, w.data_ptr(), k, m, ns, k,
                                   ex.scale.data_ptr(), sw.data_ptr(), ns, None, 0, EPILOGUES["separate"],
                                   y.data_ptr(), nat.F16, ns, stream), "b2_qgemm")
            lo, hi = rng
            a, b = shard_overlap(c0, ns, lo, hi)
            ex.exchange_slice(y.data_ptr() + (a - c0) * 2 if b > a else y.data_ptr(), m, b - a, ns,
                              _block(self.block, hi - lo), 1 - cur, a - lo, stream)
            cur = 1 - cur
        raise AssertionError("unreachable")

    def forward(self, x):
        if self.activations == "int8":
            return self._forward_int8(x)
        h = self.hidden
        for qkv_l, out_l, up_l, down_l in self.layers:
            qkv = qkv_l(x)
            o = out_l(qkv[:, :h])
            x = down_l(up_l(o))
        return x

    __call__ = forward
