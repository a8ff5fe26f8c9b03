"""GPU parity of the MoE grouping (b2sq_moe_sorting) and the grouped per-expert
int8 GEMM (b2sq_gemm_i8_grouped) against the oracle, and the whole config-5
pipeline: route -> sort -> MoE smoothquant into expert order -> grouped GEMM."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu


def to_np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("T,E,K,unit", [(4096, 8, 2, 1), (3328, 32, 5, 32), (3328, 64, 5, 16), (100, 8, 2, 4),
                                        (1, 4, 1, 1), (5000, 1024, 3, 1)])
def test_moe_sorting_parity(cuda_device, T, E, K, unit):
    rng = np.random.default_rng(T + E)
    ids = synth.topk_routing_np(rng, T, E, K) if K <= E else rng.integers(0, E, (T, K)).astype(np.int32)
    ids[T // 3, 0] = -1
    ids[T // 2, K - 1] = E + 3  # invalid ids are skipped (rocwmma_moe_sorting.cpp:70, :120)
    cnt, start, sids, perm = api.moe_sorting(torch.from_numpy(ids).to(cuda_device), E, unit)
    torch.cuda.synchronize()
    c0, s0, sid0, p0 = O.moe_sorting(ids, E, unit)
    assert np.array_equal(to_np(cnt), c0)
    assert np.array_equal(to_np(start), s0)
    total = int(s0[-1])
    assert np.array_equal(to_np(sids)[:total], sid0[:total])
    assert np.array_equal(to_np(perm), p0)
    # the reference's contract independent of order: each segment holds exactly its tokens
    for e in range(min(E, 16)):
        seg = to_np(sids)[s0[e]:s0[e] + c0[e]]
        assert sorted(seg.tolist()) == sorted(np.repeat(np.arange(T), (ids == e).sum(1)).tolist())


@pytest.mark.parametrize("counts,N,K", [([300, 0, 129, 1, 700, 128, 5, 256], 512, 1024),
                                        ([64, 64], 300, 256), ([1000], 1000, 1000 + 24)])
def test_grouped_gemm_parity(cuda_device, counts, N, K):
    dev = cuda_device
    rng = np.random.default_rng(len(counts) * 7 + N)
    E = len(counts)
    start = np.zeros(E + 1, np.int32)
    pad = 16
    for g, c in enumerate(counts):
        start[g + 1] = start[g] + ((c + pad - 1) // pad) * pad  # padded segments, like the sorter
    rows = int(start[-1]) + 37
    Kp = ((K + 15) // 16) * 16
    a = np.zeros((rows, Kp), np.int8)
    a[:, :K] = synth.weights_np(rng, rows, K)
    w = np.zeros((E, N, Kp), np.int8)
    w[:, :, :K] = synth.weights_np(rng, E * N, K).reshape(E, N, K)
    sa = synth.scales_np(rng, rows)
    sb = synth.scales_np(rng, E * N)
    cnt = np.array(counts, np.int32)
    ta = torch.from_numpy(a).to(dev)[:, :K]
    tw = torch.from_numpy(w).to(dev)[:, :, :K]
    st_, ct_ = torch.from_numpy(start).to(dev), torch.from_numpy(cnt).to(dev)
    acc = api.gemm_grouped(ta, tw, st_, ct_, out_dtype=torch.int32)
    out = api.gemm_grouped(ta, tw, st_, ct_, torch.from_numpy(sa).to(dev), torch.from_numpy(sb).to(dev),
                           out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    acc0, out0 = O.gemm_grouped(a[:, :K], w[:, :, :K], start, cnt, sa, sb, "bf16")
    assert np.array_equal(to_np(acc), acc0)  # rows outside the groups stay 0 (zero-initialised c)
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), out0)


def test_moe_pipeline_c5(cuda_device):
    """Config 5: 4096 tokens x 4096 hidden, 8 experts, top-2 routing from softmax
    of N(0,1) logits, per-expert smooth scales, per-expert W [14336, 4096]."""
    dev = cuda_device
    T, H, E, K, N = synth.MOE_TOKENS, synth.MOE_HIDDEN, synth.MOE_EXPERTS, synth.MOE_TOPK, synth.MOE_INTER
    rng = np.random.default_rng(synth.MOE_SEED)
    x = synth.activations_np(rng, T, H, 0, 1.0)
    s = synth.smooth_np(rng, H, E)
    ids = synth.topk_routing_np(rng, T, E, K)
    w = synth.torch_int8_uniform((E, N, H), dev, 51)
    sb = synth.torch_scales(E * N, dev, 52)
    tids = torch.from_numpy(ids).to(dev)
    cnt, start, _, perm = api.moe_sorting(tids, E, 1)
    qy, rs = api.moe_smoothquant(torch.from_numpy(x).to(dev), torch.from_numpy(s).to(dev), tids, row_perm=perm,
                                 out_rows=T * K)
    out = api.gemm_grouped(qy, w, start, cnt, rs, sb, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    # oracle: quantise in the reference's order, then per (token, slot) GEMM with its expert
    q0, r0 = O.moe_smoothquant(x, s, ids)
    p = to_np(perm)
    assert np.array_equal(to_np(qy)[p], q0) and np.array_equal(to_np(rs)[p], r0)
    wn = w.cpu().numpy()
    sbn = sb.cpu().numpy()
    flat_e = ids.reshape(-1)
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    for e in range(E):
        fl = np.nonzero(flat_e == e)[0][::7]  # a sample of every expert's rows
        acc = O.gemm_i8_acc(np.ascontiguousarray(q0[fl]), wn[e].T)
        ref = O.dequant(acc, r0[fl], sbn[e * N:(e + 1) * N], out_dtype="bf16")
        assert np.array_equal(got[p[fl]], ref), f"expert {e}"
