"""N-sharded (column-parallel) smoothquant -> int8 GEMM across the GPUs of one node.

The GEMM shards naturally along N: rank r owns the weight rows
W[n0:n1, :] (K-major) and their per-channel scales.  One process per GPU,
torch.distributed (NCCL on GPUs) for the exchange steps:

  1. quantise the activations: with ``x_source="replicated"`` every rank
     holds x and quantises it itself (no communication; quantising is
     cheaper than moving Xq); with ``x_source="rank0"`` rank 0 quantises and
     broadcasts Xq (int8, half the bytes of fp16 x) and the row scales;
  2. each rank runs the GEMM on its N shard (no communication);
  3. optionally all-gather the output shards into the full row-major [M, N]
     (``gather_output=True``); otherwise the output stays N-sharded, as a
     column-parallel layer's output normally does.

The compute steps are injected (``ops``) so the same host logic runs with the
library's CUDA kernels on GPUs and with a CPU implementation on ``gloo`` ranks
in the tests.  There is no equivalent in the reference (single GPU only).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

SHARD_ALIGN = 256  # shard widths are multiples of the GEMM tile width


def shard_range(n: int, world: int, rank: int, align: int = SHARD_ALIGN) -> tuple[int, int]:
    """[n0, n1) of rank's N shard: equal multiples of `align`, the remainder on the last ranks' tail."""
    units = (n + align - 1) // align
    per, extra = divmod(units, world)
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    return min(n, u0 * align), min(n, u1 * align)


@dataclass
class Ops:
    """Compute steps: smoothquant(x, s) -> (xq, row_scale); gemm(xq, w_shard_nk, sa, sb) -> out."""
    smoothquant: Callable
    gemm: Callable


def cuda_ops(out_dtype: torch.dtype = torch.bfloat16) -> Ops:
    from . import api

    ws = api.Workspace()
    return Ops(
        smoothquant=lambda x, s: api.smoothquant(x, s),
        gemm=lambda xq, w, sa, sb: api.gemm_quant(xq, w.t(), sa, sb, out_dtype=out_dtype, workspace=ws),
    )


class ShardedPrefill:
    """Column-parallel quantised linear layer over the ranks of a process group."""

    def __init__(self, w_shard_nk: torch.Tensor, sb_shard: torch.Tensor, n_total: int, ops: Ops,
                 group: Optional[dist.ProcessGroup] = None):
        self.w = w_shard_nk
        self.sb = sb_shard
        self.n_total = n_total
        self.ops = ops
        self.group = group
        # Without an initialised process group the layer is a single shard.
        self.dist = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.dist else 1
        self.rank = dist.get_rank(group) if self.dist else 0
        self.shards = [shard_range(n_total, self.world, r) for r in range(self.world)]
        assert self.w.shape[0] == self.shards[self.rank][1] - self.shards[self.rank][0]

    def quantize(self, x: Optional[torch.Tensor], smooth: torch.Tensor, x_source: str, m: int, k: int):
        if x_source == "replicated" or self.world == 1:
            return self.ops.smoothquant(x, smooth)
        if x_source != "rank0":
            raise ValueError("x_source must be 'replicated' or 'rank0'")
        dev = smooth.device
        if self.rank == 0:
            xq, rs = self.ops.smoothquant(x, smooth)
        else:
            xq = torch.empty((m, k), dtype=torch.int8, device=dev)
            rs = torch.empty((m,), dtype=torch.float32, device=dev)
        dist.broadcast(xq.view(torch.uint8), 0, group=self.group)  # byte view: every backend moves uint8
        dist.broadcast(rs, 0, group=self.group)
        return xq, rs

    def gather(self, out_shard: torch.Tensor) -> torch.Tensor:
        """All-gather the N shards into a row-major [M, N] tensor."""
        if self.world == 1:
            return out_shard
        m = out_shard.shape[0]
        widths = [b - a for a, b in self.shards]
        if len(set(widths)) == 1 and dist.get_backend(self.group) == "nccl":
            buf = torch.empty((self.world, m, widths[0]), dtype=out_shard.dtype, device=out_shard.device)
            dist.all_gather_into_tensor(buf, out_shard.contiguous(), group=self.group)
            return buf.permute(1, 0, 2).reshape(m, self.n_total)
        # Unequal shards (or a backend without all_gather_into_tensor): pad
        # every shard to the widest, gather byte views, crop.
        wmax = max(widths)
        mine = torch.zeros((m, wmax), dtype=out_shard.dtype, device=out_shard.device)
        mine[:, :out_shard.shape[1]] = out_shard
        parts = [torch.empty((m, wmax), dtype=out_shard.dtype, device=out_shard.device) for _ in widths]
        dist.all_gather([p.view(torch.uint8) for p in parts], mine.view(torch.uint8), group=self.group)
        return torch.cat([p[:, :w_] for p, w_ in zip(parts, widths)], dim=1)

    def forward(self, x: Optional[torch.Tensor], smooth: torch.Tensor, m: int, k: int,
                x_source: str = "replicated", gather_output: bool = False) -> torch.Tensor:
        xq, rs = self.quantize(x, smooth, x_source, m, k)
        out = self.ops.gemm(xq, self.w, rs, self.sb)
        return self.gather(out) if gather_output else out
