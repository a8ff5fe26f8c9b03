"""GPU parity of the smoothquant kernels against the CPU oracle: int8 output
and fp32 row scales bit-exact.  Calls go through the C ABI (libb2sq.so)."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu


def run_sq(x_np, s_np, qmax=127.0, offset=0):
    dev = torch.device("cuda", 0)
    M, N = x_np.shape
    if offset:  # deliberately misaligned x / y (the generic path)
        xb = torch.zeros(M * N + offset, dtype=torch.float16, device=dev)
        xb[offset:] = torch.from_numpy(x_np.reshape(-1)).to(dev)
        x = xb[offset:].view(M, N)
    else:
        x = torch.from_numpy(x_np).to(dev)
    s = torch.from_numpy(s_np).to(dev)
    y, rs = api.smoothquant(x, s, qmax)
    torch.cuda.synchronize()
    return y.cpu().numpy(), rs.cpu().numpy()


def check_sq(x, s, qmax=127.0, offset=0):
    y, rs = run_sq(x, s, qmax, offset)
    y0, rs0 = O.smoothquant(x, s, qmax)
    assert np.array_equal(rs.view(np.uint32), rs0.view(np.uint32)), "row_scale mismatch"
    assert np.array_equal(y, y0), f"int8 mismatch at {np.argwhere(y != y0)[:5]}"


def test_kat_reference_inputs(cuda_device):
    M, N = 3328, 4096  # rocwmma_smoothquant.cpp:170 defaults, x = 0.5, s = 1 (:140-141)
    y, rs = run_sq(np.full((M, N), 0.5, np.float16), np.ones(N, np.float32))
    assert np.all(y == 127) and np.all(rs == np.float32(0.5) / np.float32(127))


@pytest.mark.parametrize("M,N", [(256, 1024), (16, 8192), (64, 8192), (333, 4096), (17, 2048), (9, 256),
                                 (4, 64), (3, 8), (31, 16384), (2, 12288), (5, 10000)])
def test_vector_path(cuda_device, M, N):
    rng = np.random.default_rng(M + N)
    check_sq(synth.activations_np(rng, M, N, 8, 20.0), synth.smooth_np(rng, N))


@pytest.mark.parametrize("M,N", [(7, 1000 + 3), (5, 7), (4, 24577), (3, 40000), (1, 1)])
def test_generic_path(cuda_device, M, N):
    rng = np.random.default_rng(M * 7 + N)
    check_sq(synth.activations_np(rng, M, N, min(8, N), 30.0), synth.smooth_np(rng, N))


def test_misaligned_pointer(cuda_device):
    rng = np.random.default_rng(1)
    check_sq(synth.activations_np(rng, 6, 512, 4, 20.0), synth.smooth_np(rng, 512), offset=1)


def test_zero_rows_ties_and_qmax(cuda_device):
    rng = np.random.default_rng(2)
    x = synth.activations_np(rng, 8, 1024, 8, 20.0)
    x[3] = 0
    x[5, :8] = np.array([127, 2.5, 3.5, -2.5, -3.5, 0.5, 1.5, -0.5], np.float16)
    x[5, 8:] = 0
    s = np.ones(1024, np.float32)
    check_sq(x, s)
    check_sq(x, s, qmax=7.0)
    y, rs = run_sq(x, s)
    assert rs[3] == 0 and np.all(y[3] == 0)
    assert list(y[5, :8]) == [127, 2, 4, -2, -4, 0, 2, 0]


def test_c1_golden(cuda_device):
    from golden.make_golden import GOLDEN

    g = np.load(GOLDEN)
    y, rs = run_sq(g["x"], g["smooth"])
    assert np.array_equal(y, g["y"]) and np.array_equal(rs, g["row_scale"])


def test_full_size_prefill_rows(cuda_device):
    """C4 activation shape 16384 x 8192 on the device; whole output checked
    against the oracle, plus a size-independent property."""
    dev = cuda_device
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    M, N = 16384, 8192
    x = (torch.randn((M, N), generator=g, device=dev) * 2).to(torch.float16)
    s = torch.empty((N,), device=dev).uniform_(0.5, 2.0, generator=g)
    y, rs = api.smoothquant(x, s)
    torch.cuda.synchronize()
    # properties: every row reaches +-127 exactly once its absmax column is hit
    assert int(y.abs().amax(dim=1).min()) == 127
    y0, rs0 = O.smoothquant(x.cpu().numpy(), s.cpu().numpy())  # every row (near-ties included)
    assert np.array_equal(y.cpu().numpy(), y0)
    assert np.array_equal(rs.cpu().numpy(), rs0)


def test_bad_args_raise(cuda_device):
    x = torch.zeros((4, 64), dtype=torch.float16, device=cuda_device)
    s = torch.ones(64, device=cuda_device)
    with pytest.raises(api.B2sqError):
        api.smoothquant(x, s, quant_max=0.0)
    with pytest.raises(api.B2sqError):
        api.smoothquant(x, s, quant_max=200.0)


@pytest.mark.parametrize("qmax", [127.0, 100.0, 7.0, 100.5, 126.9])
def test_special_values_and_qmax(cuda_device, qmax):
    """NaN / +-inf / subnormal / huge inputs and integral or fractional quant_max:
    the fast rounding path (integral qmax) and the exact path must both match."""
    rng = np.random.default_rng(int(qmax * 10))
    M, N = 12, 2048
    x = synth.activations_np(rng, M, N, 8, 20.0)
    x[0, 3] = np.inf
    x[1, 7] = -np.inf
    x[2, 11] = np.nan
    x[3, :] = np.float16(6e-8)       # subnormal fp16 everywhere
    x[4, :] = 0
    x[4, 100] = np.float16(65504)    # max fp16
    x[5, 200] = np.nan
    x[5, 201] = np.inf
    s = synth.smooth_np(rng, N)
    s[9] = 1e-30                     # tiny scale: subnormal products
    check_sq(x, s, qmax)
    check_sq(x[:, :1000].copy(), s[:1000].copy(), qmax)  # generic (unaligned-N) path too


@pytest.mark.parametrize("qmax", [127.0, 100.5])
def test_special_values_streaming_path(cuda_device, qmax):
    """Rows of 8192+ elements in inputs of >= 2^24 elements take the TMA-staged
    kernel; rows with NaN, +-inf, overflow to inf after smoothing, or
    all-subnormal values take its exact (clamped) branch, ordinary rows its
    fast branch.  All bit-exact."""
    rng = np.random.default_rng(77)
    M, N = 2050, 8200  # 2050 x 8192 >= 2^24 elements; N = 8200: rows not a multiple of 16 bytes
    x = synth.activations_np(rng, M, N, 8, 20.0)
    s = synth.smooth_np(rng, N)
    x[10, 5] = np.nan
    x[11, 6] = np.inf
    x[12, 7] = -np.inf
    x[13, :] = np.float16(6e-8)
    x[14, :] = 0
    x[15, 3] = np.float16(60000)
    s[3] = 1e38                       # x[15,3] * s[3] overflows fp32 -> inf
    x[16, 9] = np.nan
    x[16, 10] = np.inf
    check_sq(x[:, :8192].copy(), s[:8192].copy(), qmax)  # whole-row bulk stores
    check_sq(x, s, qmax)  # row bytes not a multiple of 16: direct stores
