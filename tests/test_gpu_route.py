"""GPU parity of the MoE router (b2sq_topk_softmax, rocwmma_topk_softmax.cpp)
against the oracle: indices and fp32 weights bit-exact, including ties, NaN /
inf logits, topk > experts and the wide (> 64 experts) variant; then the whole
device MoE pipeline from logits: route -> sort -> MoE smoothquant in expert
order -> grouped GEMM."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu


def check_route(logits, topk, sentinel=True):
    dev = torch.device("cuda", 0)
    T = logits.shape[0]
    w0 = np.full((T, topk), 7.5, np.float32) if sentinel else np.zeros((T, topk), np.float32)
    i0 = np.full((T, topk), 99, np.int32) if sentinel else np.zeros((T, topk), np.int32)
    tw, ti = torch.from_numpy(w0).to(dev), torch.from_numpy(i0).to(dev)
    api.topk_softmax(torch.from_numpy(logits).to(dev), topk, tw, ti)
    torch.cuda.synchronize()
    rw, ri = O.topk_softmax(logits, topk, w0, i0)
    got_w, got_i = tw.cpu().numpy(), ti.cpu().numpy()
    assert np.array_equal(got_i, ri), f"index mismatch at {np.argwhere(got_i != ri)[:5]}"
    # bit-exact, except that NaN encodings are the platform's own (x86 and the
    # GPU produce different default NaN bits)
    same = (got_w.view(np.uint32) == rw.view(np.uint32)) | (np.isnan(got_w) & np.isnan(rw))
    assert same.all(), f"weight bits differ at {np.argwhere(~same)[:5]}"
    return got_w, got_i


# the reference driver's configs (rocwmma_topk_softmax.cpp:250-255) plus ragged expert counts
@pytest.mark.parametrize("T,E,K", [(128, 8, 4), (3328, 8, 2), (3328, 16, 2), (3328, 32, 5), (3328, 64, 5),
                                   (1000, 1, 1), (77, 2, 2), (77, 3, 2), (500, 5, 3), (300, 20, 4), (300, 33, 6),
                                   (300, 63, 8), (200, 65, 4), (200, 128, 8), (64, 1000, 5), (5, 4096, 3)])
def test_route_parity(cuda_device, T, E, K):
    rng = np.random.default_rng(T * 100 + E)
    # the reference driver's distribution: uniform [-0.5, 0.5) (:216), in fp16
    logits = (rng.random((T, E), dtype=np.float32) - 0.5).astype(np.float16)
    check_route(logits, K)


def test_route_ties_special_values(cuda_device):
    rng = np.random.default_rng(3)
    T, E = 64, 16
    logits = rng.integers(-2, 3, (T, E)).astype(np.float16)  # many exact ties
    logits[0] = 0
    logits[1, 3] = np.nan
    logits[2, :] = -np.inf
    logits[3, 5] = np.inf
    logits[4, 0] = np.nan  # NaN in lane 0 stays the first pick
    logits[5] = np.float16(65504)
    logits[6, ::2] = -np.inf
    w, i = check_route(logits, 6)
    assert i[0].tolist()[:3] == [0, 8, 4]  # tree order for 16 equal logits
    check_route(logits[:, :13].copy(), 20)  # topk > experts: the tail slots stay untouched
    wide = rng.integers(-2, 3, (16, 200)).astype(np.float16)
    wide[1, 10] = np.nan
    wide[2, :] = -np.inf
    check_route(wide, 70)  # more rounds than the 64 candidates: (-1, -1) slots


def test_route_empty_and_bad_args(cuda_device):
    x = torch.zeros((0, 8), dtype=torch.float16, device=cuda_device)
    w, i = api.topk_softmax(x, 2)
    assert w.shape == (0, 2)
    with pytest.raises(ValueError):
        api.topk_softmax(torch.zeros((4, 8), dtype=torch.float32, device=cuda_device), 2)


def test_device_moe_pipeline_from_logits(cuda_device):
    """logits -> b2sq_topk_softmax -> b2sq_moe_sorting -> MoE smoothquant into
    expert order -> grouped GEMM, every stage on the device; checked stage by
    stage against the oracle chain."""
    dev = cuda_device
    T, H, E, K, N = 1024, 2048, 8, 2, 1024
    rng = np.random.default_rng(11)
    logits = rng.standard_normal((T, E), dtype=np.float32).astype(np.float16)
    x = synth.activations_np(rng, T, H, 4, 10.0)
    s = synth.smooth_np(rng, H, E)
    w = synth.torch_int8_uniform((E, N, H), dev, 61)
    sb = synth.torch_scales(E * N, dev, 62)

    tw, ti = api.topk_softmax(torch.from_numpy(logits).to(dev), K)
    cnt, start, _, perm = api.moe_sorting(ti, E, 16)
    qy, rs = api.moe_smoothquant(torch.from_numpy(x).to(dev), torch.from_numpy(s).to(dev), ti, row_perm=perm,
                                 out_rows=int(start[-1].item()))
    out = api.gemm_grouped(qy, w, start, cnt, rs, sb, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()

    w0, i0 = O.topk_softmax(logits, K)
    assert np.array_equal(ti.cpu().numpy(), i0) and np.array_equal(tw.cpu().numpy(), w0)
    c0, s0, _, p0 = O.moe_sorting(i0, E, 16)
    assert np.array_equal(cnt.cpu().numpy(), c0) and np.array_equal(perm.cpu().numpy(), p0)
    q0, r0 = O.moe_smoothquant(x, s, i0)
    assert np.array_equal(qy.cpu().numpy()[p0], q0) and np.array_equal(rs.cpu().numpy()[p0], r0)
    wn, sbn = w.cpu().numpy(), sb.cpu().numpy()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    flat_e = i0.reshape(-1)
    for e in range(E):
        fl = np.nonzero(flat_e == e)[0][::5]
        acc = O.gemm_i8_acc(np.ascontiguousarray(q0[fl]), wn[e].T)
        ref = O.dequant(acc, r0[fl], sbn[e * N:(e + 1) * N], out_dtype="bf16")
        assert np.array_equal(got[p0[fl]], ref), f"expert {e}"
