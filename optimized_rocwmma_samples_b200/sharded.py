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
     (``gather_output=True``: GEMM, then NCCL all-gather, or
     ``gather_output="fused"``: one GEMM whose epilogue stores every output
     tile into all ranks' [M, N] buffers over NVLink, b2sq_gemm_i8_allgather);
     otherwise the output stays N-sharded, as a column-parallel layer's
     output normally does.

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
    """Compute steps: smoothquant(x, s) -> (xq, row_scale); gemm(xq, w_shard_nk, sa, sb) -> out;
    gemm_gather(xq, w_shard_nk, sa, sb, n0, n_total, layer) -> the gathered [M, n_total] output."""
    smoothquant: Callable
    gemm: Callable
    gemm_gather: Optional[Callable] = None
    close: Callable = lambda: None  # releases buffers / peer mappings the steps created


class PeerOutput:
    """A row-major [M, N] output buffer on every rank, each mapped into every
    other rank's process by CUDA IPC, so one GEMM epilogue can store its shard
    into all of them.  Collective to create (handles travel by
    all_gather_object); close() unmaps the peers' buffers."""

    def __init__(self, m: int, n_total: int, dtype: torch.dtype, device: torch.device, group, world: int, rank: int):
        from . import api

        self.local = torch.empty((m, n_total), dtype=dtype, device=device)
        mine = api.ipc_export(self.local)
        every = [None] * world
        dist.all_gather_object(every, mine, group=group)
        self.bases, self.ptrs = [], []
        for r, (handle, offset) in enumerate(every):
            if r == rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                base = api.ipc_open(handle)
                self.bases.append(base)
                self.ptrs.append(base + offset)

    def close(self):
        from . import api

        for b in self.bases:
            api.ipc_close(b)
        self.bases, self.ptrs = [], []


class MulticastOutput:
    """A row-major [M, N] output buffer in torch symmetric memory on every
    rank, with the NVSwitch multicast view that maps all ranks' buffers: one
    multimem store reaches every rank.  Collective to create; raises if the
    devices have no multicast support."""

    def __init__(self, m: int, n_total: int, dtype: torch.dtype, device: torch.device, group):
        import torch.distributed._symmetric_memory as symm

        self.local = symm.empty((m, n_total), dtype=dtype, device=device)
        self.handle = symm.rendezvous(self.local, group if group is not None else dist.group.WORLD)
        mc = int(self.handle.multicast_ptr)
        if mc == 0:
            raise RuntimeError("no NVSwitch multicast mapping for this buffer")
        base = int(self.handle.buffer_ptrs[self.handle.rank])
        self.mc = mc + (self.local.data_ptr() - base)


def multicast_supported(device: torch.device) -> bool:
    try:
        from torch._C._distributed_c10d import _SymmetricMemory
        from torch.distributed._symmetric_memory import DeviceType

        return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index or 0))
    except Exception:  # an older torch, or no symmetric memory support
        return False


def cuda_ops(out_dtype: torch.dtype = torch.bfloat16, gather: str = "auto") -> Ops:
    """The quantised activations, row scales and GEMM output live in buffers
    kept per shape and reused by the next call of the same shape (as a layer's
    workspace would be): a returned tensor is valid until that next call.

    gather: how the fused GEMM + all-gather reaches the other ranks --
    "multicast" (NVSwitch multimem stores, one copy per output piece),
    "ipc" (plain stores into every peer's buffer), or "auto" (= "ipc", the
    faster of the two at 2 and at 8 GPUs)."""
    from . import api

    if gather not in ("auto", "multicast", "ipc"):
        raise ValueError("gather must be 'auto', 'multicast' or 'ipc'")
    ws = api.Workspace()
    peers: dict = {}
    flag: dict = {}

    def barrier(layer, dev):
        # one-element all-reduce on the current stream: ordered after this
        # rank's kernels, complete only once every rank has reached it
        if dev not in flag:
            flag[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.all_reduce(flag[dev], group=layer.group)

    def gemm_gather(xq, w, sa, sb, n0, n_total, layer):
        m, n = xq.shape[0], w.shape[0]
        dev = xq.device
        # the same choice on every rank (the buffers are created collectively)
        fits = m > 128 and all((b - a) % 64 == 0 for a, b in layer.shards)
        # auto = ipc: an all-gather is bound by what every GPU must RECEIVE ((world-1)/world of the
        # output), which multicast does not reduce; measured at 8 GPUs (config 4) 1.42 ms with
        # peer stores, 1.46 ms with multimem; at 2 GPUs 1.39 vs 1.66 ms
        use_mc = fits and gather == "multicast" and multicast_supported(dev)
        key = (m, n_total, dev, use_mc)
        if key not in peers:
            peers[key] = (MulticastOutput(m, n_total, out_dtype, dev, layer.group) if use_mc else
                          PeerOutput(m, n_total, out_dtype, dev, layer.group, layer.world, layer.rank))
        po = peers[key]
        barrier(layer, dev)  # every rank is done with the previous contents
        if use_mc:
            api.gemm_allgather_mc(xq, w.t(), po.local.data_ptr(), po.mc, n0, n_total, sa, sb, out_dtype=out_dtype,
                                  workspace=ws)
        else:
            api.gemm_allgather(xq, w.t(), po.ptrs, layer.rank, n0, n_total, sa, sb, out_dtype=out_dtype, workspace=ws)
        barrier(layer, dev)  # every shard has landed in every buffer
        return po.local

    def close():
        torch.cuda.synchronize()
        for po in peers.values():
            if isinstance(po, PeerOutput):
                po.close()
        peers.clear()
        bufs.clear()

    bufs: dict = {}  # per-shape activation and output buffers, reused by later calls

    def buf(key, shape, dtype, dev):
        k = (key, tuple(shape), dtype, dev)
        if k not in bufs:
            bufs[k] = torch.empty(shape, dtype=dtype, device=dev)
        return bufs[k]

    def smoothquant(x, s):
        m, k = x.shape
        return api.smoothquant(x, s, y=buf("xq", (m, k), torch.int8, x.device),
                               row_scale=buf("rs", (m,), torch.float32, x.device))

    def gemm(xq, w, sa, sb):
        c = buf("out", (xq.shape[0], w.shape[0]), out_dtype, xq.device)
        return api.gemm_quant(xq, w.t(), sa, sb, out_dtype=out_dtype, c=c, workspace=ws)

    return Ops(
        smoothquant=smoothquant,
        gemm=gemm,
        gemm_gather=gemm_gather,
        close=close,
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

    def gather(self, out_shard: torch.Tensor, blocked: bool = False) -> torch.Tensor:
        """All-gather the N shards.  blocked=False: a row-major [M, N] tensor;
        blocked=True (equal shard widths only): the shards as they arrive,
        [world, M, width], with no re-layout copy after the collective."""
        if self.world == 1:
            return out_shard.unsqueeze(0) if blocked else out_shard
        m = out_shard.shape[0]
        widths = [b - a for a, b in self.shards]
        if blocked and len(set(widths)) != 1:
            raise ValueError("a blocked gather needs equal shard widths")
        if len(set(widths)) == 1 and dist.get_backend(self.group) == "nccl":
            buf = torch.empty((self.world, m, widths[0]), dtype=out_shard.dtype, device=out_shard.device)
            dist.all_gather_into_tensor(buf, out_shard.contiguous(), group=self.group)
            return buf if blocked else buf.permute(1, 0, 2).reshape(m, self.n_total)
        # Unequal shards (or a backend without all_gather_into_tensor): pad
        # every shard to the widest, gather byte views, crop.
        wmax = max(widths)
        mine = torch.zeros((m, wmax), dtype=out_shard.dtype, device=out_shard.device)
        mine[:, :out_shard.shape[1]] = out_shard
        parts = [torch.empty((m, wmax), dtype=out_shard.dtype, device=out_shard.device) for _ in widths]
        dist.all_gather([p.view(torch.uint8) for p in parts], mine.view(torch.uint8), group=self.group)
        if blocked:
            return torch.stack(parts)
        return torch.cat([p[:, :w_] for p, w_ in zip(parts, widths)], dim=1)

    def forward(self, x: Optional[torch.Tensor], smooth: torch.Tensor, m: int, k: int,
                x_source: str = "replicated", gather_output=False) -> torch.Tensor:
        """gather_output: False (N-sharded result), True (GEMM then all-gather
        into [M, N]), "blocked" (GEMM then all-gather, shards left as
        [world, M, width]) or "fused" (the GEMM's epilogue gathers; the
        returned buffer is reused by the next fused call of the same shape)."""
        xq, rs = self.quantize(x, smooth, x_source, m, k)
        if gather_output == "fused" and self.world > 1:
            if self.ops.gemm_gather is None:
                raise ValueError("these ops have no fused GEMM + all-gather step")
            return self.ops.gemm_gather(xq, self.w, rs, self.sb, self.shards[self.rank][0], self.n_total, self)
        out = self.ops.gemm(xq, self.w, rs, self.sb)
        if gather_output == "blocked":
            return self.gather(out, blocked=True)
        return self.gather(out) if gather_output else out
