"""GPU parity of b2sq_smoothquant_gemm_i8 (smoothquant -> GEMM in one call,
GEMM launched with programmatic dependent launch) against the separate calls
and the oracle: int8 Xq and row scales bit-exact, fp16/bf16 output within
1 ulp (identical in practice)."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N,dt", [(16, 8192, 28672, torch.float16), (64, 8192, 28672, torch.float16),
                                      (1, 1024, 4096, torch.bfloat16), (300, 1024, 768, torch.bfloat16),
                                      (2048, 4096, 4096, torch.bfloat16)])
def test_fused_matches_separate_and_oracle(cuda_device, M, K, N, dt):
    dev = cuda_device
    rng = np.random.default_rng(M + N)
    x = torch.from_numpy(synth.activations_np(rng, M, K, 8, 30.0)).to(dev)
    s = torch.from_numpy(synth.smooth_np(rng, K)).to(dev)
    w = synth.torch_int8_uniform((N, K), dev, 7)
    sb = synth.torch_scales(N, dev, 8)
    for rep in range(2):  # repeated calls (workspace reuse, PDL twice in a row)
        c, xq, rs = api.smoothquant_gemm(x, s, w, sb, out_dtype=dt)
        y2, rs2 = api.smoothquant(x, s)
        c2 = api.gemm_quant(y2, w.t(), rs2, sb, out_dtype=dt)
        torch.cuda.synchronize()
        assert torch.equal(xq, y2) and torch.equal(rs, rs2)
        assert torch.equal(c.view(torch.int16), c2.view(torch.int16))
    y0, r0 = O.smoothquant(x.cpu().numpy(), s.cpu().numpy())
    assert np.array_equal(xq.cpu().numpy(), y0) and np.array_equal(rs.cpu().numpy(), r0)
    rows = np.arange(0, M, max(1, M // 8))
    acc = O.gemm_i8_acc(np.ascontiguousarray(y0[rows]), w.cpu().numpy().T)
    ref = O.dequant(acc, r0[rows], sb.cpu().numpy(), out_dtype="f16" if dt == torch.float16 else "bf16")
    assert np.array_equal(c[rows].view(torch.int16).cpu().numpy().view(np.uint16), ref)
    assert api.last_device_error() == 0


def test_fused_decode_replays_in_a_cuda_graph(cuda_device):
    """The fused decode call (smoothquant -> GEMM chained by programmatic
    dependent launch) captures into a CUDA graph; replays with new input
    values in the captured buffers give the results of direct calls."""
    from optimized_rocwmma_samples_b200 import api, synth

    dev = cuda_device
    M, K, N = 16, 4096, 8192
    w = synth.torch_int8_uniform((N, K), dev, 41)
    sb = synth.torch_scales(N, dev, 42)
    s = torch.empty((K,), device=dev).uniform_(0.5, 2.0)
    x = torch.empty((M, K), dtype=torch.float16, device=dev)
    y = torch.empty((M, K), dtype=torch.int8, device=dev)
    r = torch.empty((M,), dtype=torch.float32, device=dev)
    o = torch.empty((M, N), dtype=torch.float16, device=dev)
    ws = api.Workspace()

    def step():
        api.smoothquant_gemm(x, s, w, sb, out_dtype=torch.float16, xq=y, row_scale=r, c=o, workspace=ws)

    x.copy_(torch.randn((M, K), device=dev).to(torch.float16))
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        step()  # first call outside capture: one-time attribute setup
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
    for seed in range(3):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        x.copy_((torch.randn((M, K), generator=g, device=dev) * 2).to(torch.float16))
        graph.replay()
        torch.cuda.synchronize()
        got = o.clone()
        ref, _, _ = api.smoothquant_gemm(x, s, w, sb, out_dtype=torch.float16, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


@pytest.mark.parametrize("M,K,N,qmax", [(16, 1040, 4096, 127.0), (3, 8192, 28672, 127.0), (11, 4112, 2304, 100.5),
                                        (16, 2048, 512, 7.0), (1, 16, 256, 127.0)])
def test_decode_edge_cases_match_two_calls(cuda_device, M, K, N, qmax):
    """Decode sizes through the one-call entry: Xq, row scales and the fp16
    output are bit-identical to b2sq_smoothquant followed by b2sq_gemm_i8,
    including ragged K, fractional quant_max and rows with inf / NaN /
    all-zero inputs."""
    dev = cuda_device
    rng = np.random.default_rng(M * 7 + K)
    xn = synth.activations_np(rng, M, K, 4, 30.0)
    if M >= 3:
        xn[0, K // 3] = np.inf
        xn[1, :] = 0
        xn[2, 5] = np.nan
    x = torch.from_numpy(xn).to(dev)
    s = torch.from_numpy(synth.smooth_np(rng, K)).to(dev)
    w = synth.torch_int8_uniform((N, K), dev, 9)
    sb = synth.torch_scales(N, dev, 10)
    for rep in range(2):
        c, xq, rs = api.smoothquant_gemm(x, s, w, sb, quant_max=qmax, out_dtype=torch.float16)
        y2, rs2 = api.smoothquant(x, s, quant_max=qmax)
        c2 = api.gemm_quant(y2, w.t(), rs2, sb, out_dtype=torch.float16)
        torch.cuda.synchronize()
        assert torch.equal(xq, y2)
        assert torch.equal(rs.view(torch.int32), rs2.view(torch.int32)) or \
            bool(((rs == rs2) | (torch.isnan(rs) & torch.isnan(rs2))).all())
        assert torch.equal(c.view(torch.int16), c2.view(torch.int16))
    y0, r0 = O.smoothquant(xn, s.cpu().numpy(), qmax)
    assert np.array_equal(xq.cpu().numpy(), y0)
    assert api.last_device_error() == 0
