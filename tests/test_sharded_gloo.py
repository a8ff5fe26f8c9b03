"""The N-sharded multi-GPU host logic on CPU: two `gloo` ranks run
ShardedPrefill with the CPU oracle as the compute step and must reproduce the
single-process result exactly (replicated and rank-0-broadcast activations,
sharded and gathered outputs).  No GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from optimized_rocwmma_samples_b200.sharded import Ops, ShardedPrefill, shard_range

M, K, N = 64, 256, 1280  # N = 5 tile widths: unequal shards over 2 ranks


def inputs():
    from optimized_rocwmma_samples_b200 import synth

    rng = np.random.default_rng(5)
    x = synth.activations_np(rng, M, K, 4, 20.0)
    s = synth.smooth_np(rng, K)
    w = synth.weights_np(rng, N, K)  # [N, K] K-major
    sb = synth.scales_np(rng, N)
    return x, s, w, sb


def oracle_ops():
    import oracle as O

    def sq(x, s):
        y, rs = O.smoothquant(x.numpy(), s.numpy())
        return torch.from_numpy(y), torch.from_numpy(rs)

    def gemm(xq, w, sa, sb):
        acc = O.gemm_i8_acc(xq.numpy(), w.numpy().T)
        bits = O.dequant(acc, sa.numpy(), sb.numpy(), out_dtype="bf16")
        return torch.from_numpy(bits.view(np.int16))

    # the fused GEMM + all-gather step, restated as GEMM then gather (its contract)
    def gemm_gather(xq, w, sa, sb, n0, n_total, layer):
        assert layer.shards[layer.rank][0] == n0 and layer.n_total == n_total
        return layer.gather(gemm(xq, w, sa, sb))

    return Ops(smoothquant=sq, gemm=gemm, gemm_gather=gemm_gather)


def worker(rank, world, port, q):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "oracle")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, s, w, sb = inputs()
        n0, n1 = shard_range(N, world, rank)
        layer = ShardedPrefill(torch.from_numpy(w[n0:n1].copy()), torch.from_numpy(sb[n0:n1].copy()), N,
                               oracle_ops())
        out = {}
        out["repl_gather"] = layer.forward(torch.from_numpy(x), torch.from_numpy(s), M, K, "replicated", True)
        xin = torch.from_numpy(x) if rank == 0 else None
        out["rank0_gather"] = layer.forward(xin, torch.from_numpy(s), M, K, "rank0", True)
        out["rank0_shard"] = layer.forward(xin, torch.from_numpy(s), M, K, "rank0", False)
        out["repl_fused"] = layer.forward(torch.from_numpy(x), torch.from_numpy(s), M, K, "replicated", "fused")
        # equal shards (the first 1024 columns): the blocked gather keeps [world, M, width]
        e0, e1 = shard_range(1024, world, rank)
        layer_eq = ShardedPrefill(torch.from_numpy(w[e0:e1].copy()), torch.from_numpy(sb[e0:e1].copy()), 1024,
                                  oracle_ops())
        out["repl_blocked"] = layer_eq.forward(torch.from_numpy(x), torch.from_numpy(s), M, K, "replicated", "blocked")
        q.put((rank, {k: v.numpy() for k, v in out.items()}, (n0, n1)))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def test_shard_ranges():
    assert shard_range(28672, 8, 3) == (3 * 3584, 4 * 3584)
    spans = [shard_range(1280, 2, r) for r in range(2)]
    assert spans == [(0, 768), (768, 1280)]
    for n, p in [(1000, 3), (28672, 8), (256, 4), (17, 2)]:
        s = [shard_range(n, p, r) for r in range(p)]
        assert s[0][0] == 0 and s[-1][1] == n and all(s[i][1] == s[i + 1][0] for i in range(p - 1))


@pytest.mark.timeout(300)
def test_two_rank_sharded_prefill_matches_single_process():
    import oracle as O

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    x, s, w, sb = inputs()
    y, rs = O.smoothquant(x, s)
    full = O.dequant(O.gemm_i8_acc(y, w.T), rs, sb, out_dtype="bf16").view(np.int16)
    for rank, out, (n0, n1) in results:
        assert np.array_equal(out["repl_gather"], full)
        assert np.array_equal(out["rank0_gather"], full)
        assert np.array_equal(out["rank0_shard"], full[:, n0:n1])
        assert np.array_equal(out["repl_fused"], full)
        blk = out["repl_blocked"]
        assert blk.shape == (world, M, 1024 // world)
        assert np.array_equal(blk.transpose(1, 0, 2).reshape(M, 1024), full[:, :1024])
