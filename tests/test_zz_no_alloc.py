"""GPU test of b2sq_gemm_i8_no_alloc, the GEMM entry point for callers that
cannot allocate device memory (an FFI host without a device allocator, or a
server that keeps all of HBM in its own pool and must not call cudaMalloc
while serving).  It takes its stream-K scratch from a fixed array inside the
library; its results must equal b2sq_gemm_i8's with a caller workspace.

Collected last on purpose (file name), so a run that stops at the first
failure has run every other test first.  It also passes run alone."""
import ctypes as C

import numpy as np
import pytest
import torch

from optimized_rocwmma_samples_b200 import _lib, api, synth

pytestmark = pytest.mark.gpu

ULP_TOL = 1  # same fp16/bf16 tolerance as the other GEMM parity tests


def ulp_dist(a_bits, b_bits):
    def ordinal(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b)

    return np.abs(ordinal(a_bits) - ordinal(b_bits))


def no_alloc(a, w, sa, sb, out_dtype):
    """C = a @ w.t() through the C ABI entry point that allocates nothing
    (a row-major, or a column-major view such as t.t() of a [K, lda] buffer)."""
    lib = _lib.load()
    M, K = a.shape
    N = w.shape[0]
    c = torch.empty((M, N), dtype=out_dtype, device=a.device)
    code = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.int32: _lib.I32}[out_dtype]
    la, lda = (_lib.ROW_MAJOR, a.stride(0)) if a.stride(1) == 1 else (_lib.COL_MAJOR, a.stride(1))
    st = lib.b2sq_gemm_i8_no_alloc(M, N, K, a.data_ptr(), la, lda, w.data_ptr(), _lib.COL_MAJOR, K,
                                   c.data_ptr(), code, N, sa.data_ptr(), sb.data_ptr(), 1.0, 1.0,
                                   torch.cuda.current_stream().cuda_stream)
    return st, c


# (128, 8192, 8192): swapped 128-wide tiles, all stream-K (~19 MiB of scratch);
# (16, 28672, 8192): decode, no scratch needed; (8192, 8192, 1024): whole tiles.
@pytest.mark.parametrize("M,N,K", [(128, 8192, 8192), (16, 28672, 8192), (8192, 8192, 1024)])
def test_no_alloc_matches_workspace_entry_point(cuda_device, M, N, K):
    dev = cuda_device
    # the first shape must really use the static scratch, the decode shape none
    if (M, N, K) == (128, 8192, 8192):
        assert api.workspace_size(M, N, K) > 0
    if (M, N, K) == (16, 28672, 8192):
        assert api.workspace_size(M, N, K) == 0
    for call in range(2):  # two calls in a row share (and must re-clear) the scratch
        a = synth.torch_int8_uniform((M, K), dev, 100 + call)
        w = synth.torch_int8_uniform((N, K), dev, 200 + call)
        sa = synth.torch_scales(M, dev, 300 + call)
        sb = synth.torch_scales(N, dev, 400 + call)
        for dt in (torch.int32, torch.float16):
            st, c = no_alloc(a, w, sa, sb, dt)
            assert st == _lib.B2SQ_OK, _lib.load().b2sq_last_error_message()
            ref = api.gemm_quant(a, w.t(), sa, sb, out_dtype=dt)
            torch.cuda.synchronize()
            if dt == torch.int32:
                assert torch.equal(c, ref)
            else:
                d = ulp_dist(c.view(torch.int16).cpu().numpy().view(np.uint16),
                             ref.view(torch.int16).cpu().numpy().view(np.uint16))
                assert d.max() <= ULP_TOL
    assert api.last_device_error() == 0


def test_no_alloc_rejects_oversized_scratch(cuda_device):
    # 100 x 16384 x 2048 with column-major A (not swapped): 1-CTA 128 x 256 tiles, 64 of
    # them over 148 SMs, all stream-K: ~39 MiB of scratch (> 24 MiB)
    dev = cuda_device
    at = synth.torch_int8_uniform((2048, 112), dev, 1)  # A^T with a 16-aligned leading dimension
    a = at[:, :100].t()
    w = synth.torch_int8_uniform((16384, 2048), dev, 2)
    sa, sb = synth.torch_scales(100, dev, 3), synth.torch_scales(16384, dev, 4)
    need = api.workspace_size(100, 16384, 2048, api.COL_MAJOR, api.COL_MAJOR)
    assert need > 24 << 20
    st, _ = no_alloc(a, w, sa, sb, torch.float16)
    assert st == _lib.B2SQ_ERR_UNSUPPORTED
    assert b"scratch" in _lib.load().b2sq_last_error_message()
