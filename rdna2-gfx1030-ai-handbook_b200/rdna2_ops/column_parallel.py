"""Column-parallel (N-sharded) quantized linear across the GPUs of one node.

Each rank owns the weight rows [start, stop) of the output dimension N
(plus their per-channel scales and bias), receives the replicated
activations, runs the fused linear locally (rotation + per-token
quantization + tcgen05 GEMM + epilogue), and -- when the caller needs the
full output on every rank -- one NCCL all-gather over NVLink reassembles
Y[M, N].  Per-token scales depend only on the activation row, which every
rank sees whole, so the gathered result is bit-identical to the single-GPU
linear.

The reference is single-GPU (no collectives anywhere); this module is the
multi-GPU execution the north star asks for, with torch.distributed as the
plumbing (one process per GPU, NCCL backend).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .qlinear import w8a8_linear


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


class ColumnParallelLinear:
    """y = x @ W.T (+ bias), W sharded along N over `group`.

    local_fn(x2d, w_shard, w_scale_shard, bias_shard) -> y_shard computes the
    rank's columns; the default is the B200 fused linear (w8a8_linear with
    the given rotation / epilogue / kind).
    """

    def __init__(self, w_shard, w_scale_shard, bias_shard, n_total, *, group=None,
                 rotation_block=None, out_dtype=None, epilogue="separate", kind="int8",
                 local_fn=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_total = n_total
        if n_total % self.world:
            raise ValueError("N must divide evenly across ranks for the all-gather")
        if w_shard.shape[0] != n_total // self.world:
            raise ValueError("weight shard does not match N / world")
        self.w, self.sw, self.bias = w_shard, w_scale_shard, bias_shard
        self.kw = dict(rotation_block=rotation_block, out_dtype=out_dtype, epilogue=epilogue, kind=kind)
        self.local_fn = local_fn or (lambda x, w, sw, b: w8a8_linear(x, w, sw, b, **self.kw))

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

    def forward(self, x, gather=True):
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
