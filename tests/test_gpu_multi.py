"""Two GPUs, and all of them up to eight (skipped with fewer): the fused GEMM + all-gather
(through ShardedPrefill: b2sq_gemm_i8_allgather with peer buffers mapped by
CUDA IPC and plain NVLink stores, and b2sq_gemm_i8_allgather_mc with
NVSwitch multimem stores when the GPUs support multicast) must give every rank the same
[M, N] output as the single-GPU GEMM and as GEMM + NCCL all-gather, bit for
bit, over repeated calls that reuse the buffers.  One process per GPU, NCCL."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# (M, K, N): N = 2816 gives unequal 256-wide shards; M = 16 the swapped (decode) kernel; 9472 x 1024 at two
# ranks is 37 x 2 = 74 CTA-pair tiles per shard, so the pair kernel's epilogue does the gathering
SHAPES = [(512, 1024, 4096), (300, 2048, 2816), (16, 8192, 4096), (9472, 1024, 1024)]


def worker(rank, world, port, q):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "oracle")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from optimized_rocwmma_samples_b200 import api, synth
        from optimized_rocwmma_samples_b200.sharded import ShardedPrefill, cuda_ops, shard_range

        dev = torch.device("cuda", rank)
        res = []
        from optimized_rocwmma_samples_b200.sharded import multicast_supported

        modes = ["ipc"] + (["multicast"] if multicast_supported(dev) else [])
        for (M, K, N), mode in [(shape, mode) for shape in SHAPES for mode in modes]:
            ops = cuda_ops(torch.bfloat16, gather=mode)
            w = synth.torch_int8_uniform((N, K), dev, 7)  # identical on every rank (seeded)
            sb = synth.torch_scales(N, dev, 8)
            n0, n1 = shard_range(N, world, rank)
            layer = ShardedPrefill(w[n0:n1].contiguous(), sb[n0:n1].contiguous(), N, ops)
            for it in range(3):
                g = torch.Generator(device=dev)
                g.manual_seed(100 + it)
                x = (torch.randn((M, K), generator=g, device=dev) * 3).to(torch.float16)
                s = torch.empty((K,), device=dev).uniform_(0.5, 2.0, generator=g)
                fused = layer.forward(x, s, M, K, "replicated", "fused").clone()
                nccl = layer.forward(x, s, M, K, "replicated", True)
                xq, rs = api.smoothquant(x, s)
                single = api.gemm_quant(xq, w.t(), rs, sb, out_dtype=torch.bfloat16)
                torch.cuda.synchronize()
                res.append((M, K, N, it, bool(torch.equal(fused, single)), bool(torch.equal(nccl, single))))
            ops.close()  # unmaps the peers' buffers (all ranks are past their last exchange)
        q.put((rank, res, api.last_device_error(), modes))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), -1, []))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return sorted({2, min(n, 8)}) if n >= 2 else [2]


@pytest.mark.timeout(900)
@pytest.mark.parametrize("world", worlds())
def test_fused_gemm_allgather_multi_gpu(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=400) for _ in range(world)]
    for p in procs:
        p.join(60)
    for rank, res, dev_err, modes in results:
        print(f"rank {rank}: gather modes {modes}")
        assert isinstance(res, list), f"rank {rank}: {res}"
        assert dev_err == 0
        for M, K, N, it, ok_fused, ok_nccl in res:
            assert ok_fused, f"rank {rank}: fused all-gather differs at {(M, K, N)} call {it}"
            assert ok_nccl, f"rank {rank}: NCCL all-gather differs at {(M, K, N)} call {it}"
