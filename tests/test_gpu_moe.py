"""GPU parity of MoE smoothquant (per-expert smooth scales, top-k slots)
against the oracle, bit-exact, including invalid expert ids (row left
unwritten, rocwmma_moe_smoothquant.cpp:86-87) and the optional row_perm."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu


def run_moe(x, s, ids, row_perm=None, sentinel=True):
    dev = torch.device("cuda", 0)
    T, H = x.shape
    rows = ids.size
    qy0 = np.full((rows, H), 55, np.int8) if sentinel else np.zeros((rows, H), np.int8)
    rs0 = np.full((rows,), 9.0, np.float32) if sentinel else np.zeros((rows,), np.float32)
    qy = torch.from_numpy(qy0).to(dev)
    rs = torch.from_numpy(rs0).to(dev)
    perm = None if row_perm is None else torch.from_numpy(row_perm).to(dev)
    api.moe_smoothquant(torch.from_numpy(x).to(dev), torch.from_numpy(s).to(dev), torch.from_numpy(ids).to(dev),
                        qy=qy, row_scale=rs, row_perm=perm)
    torch.cuda.synchronize()
    ref_q, ref_r = O.moe_smoothquant(x, s, ids, row_perm=row_perm, qy=qy0, row_scale=rs0)
    return qy.cpu().numpy(), rs.cpu().numpy(), ref_q, ref_r


@pytest.mark.parametrize("T,H,E,K", [(64, 4096, 8, 2), (33, 8192, 64, 5), (100, 1024, 32, 5), (7, 2048, 4, 1),
                                     (5, 1000, 8, 2), (3, 20000, 4, 3)])
def test_moe_parity(cuda_device, T, H, E, K):
    rng = np.random.default_rng(T * H + E)
    x = synth.activations_np(rng, T, H, 8, 20.0)
    s = synth.smooth_np(rng, H, E)
    ids = synth.topk_routing_np(rng, T, E, K)
    ids[T // 2, 0] = -1
    ids[T - 1, K - 1] = E  # out of range
    q, r, q0, r0 = run_moe(x, s, ids)
    assert np.array_equal(r.view(np.uint32), r0.view(np.uint32))
    assert np.array_equal(q, q0)


def test_moe_row_perm(cuda_device):
    rng = np.random.default_rng(9)
    T, H, E, K = 50, 4096, 8, 2
    x = synth.activations_np(rng, T, H, 8, 20.0)
    s = synth.smooth_np(rng, H, E)
    ids = synth.topk_routing_np(rng, T, E, K)
    perm = rng.permutation(T * K).astype(np.int32)
    q, r, q0, r0 = run_moe(x, s, ids, row_perm=perm)
    assert np.array_equal(q, q0) and np.array_equal(r, r0)


def test_moe_kat_reference_inputs(cuda_device):
    # rocwmma_moe_smoothquant.cpp:203 config (3328, 4096, 8 experts, top-2), constant inputs.
    T, H, E, K = 3328, 4096, 8, 2
    rng = np.random.default_rng(42)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    q, r, _, _ = run_moe(np.full((T, H), 0.5, np.float16), np.ones((E, H), np.float32), ids, sentinel=False)
    assert np.all(q == 127) and np.all(r == np.float32(0.5) / np.float32(127))


def test_moe_c5_shape(cuda_device):
    """C5: 4096 tokens x 4096 hidden, 8 experts, top-2 from softmax routing."""
    rng = np.random.default_rng(synth.MOE_SEED)
    x = synth.activations_np(rng, synth.MOE_TOKENS, synth.MOE_HIDDEN, 0, 1.0)
    s = synth.smooth_np(rng, synth.MOE_HIDDEN, synth.MOE_EXPERTS)
    ids = synth.topk_routing_np(rng, synth.MOE_TOKENS, synth.MOE_EXPERTS, synth.MOE_TOPK)
    q, r, q0, r0 = run_moe(x, s, ids, sentinel=False)
    assert np.array_equal(q, q0) and np.array_equal(r, r0)


def test_moe_streaming_special_values(cuda_device):
    rng = np.random.default_rng(78)
    T, H, E, K = 1024, 4096, 8, 2
    x = synth.activations_np(rng, T, H, 8, 20.0)
    x[3, 5] = np.nan
    x[4, 6] = np.inf
    x[5, :] = 0
    s = synth.smooth_np(rng, H, E)
    ids = synth.topk_routing_np(rng, T, E, K)
    ids[7, 1] = 99
    q, r, q0, r0 = run_moe(x, s, ids)
    assert np.array_equal(q, q0) and np.array_equal(r.view(np.uint32), r0.view(np.uint32))
