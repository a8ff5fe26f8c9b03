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
