"""GPU parity of the tcgen05 int8 GEMM: int32 accumulators bit-exact against
the oracle (exact integer arithmetic), fp16/bf16 dequantised outputs within
1 ulp of the oracle's fp32 epilogue rounded to the output type (in practice
bit-exact: both compute cvt_rn(float(acc) * (sa * sb)) in fp32)."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import api, synth

pytestmark = pytest.mark.gpu

ULP_TOL = 1  # north-star tolerance for fp16/bf16 outputs


def to_dev(arr: np.ndarray, major: str, pad: int = 0) -> torch.Tensor:
    """Logical [R, C] int8 array as a device view with the requested memory order
    and a leading dimension rounded up to 16 (+pad)."""
    dev = torch.device("cuda", 0)
    R, C = arr.shape
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if major == "row":
        ld = ((C + 15) // 16) * 16 + pad
        buf = torch.zeros((max(R, 1), ld), dtype=torch.int8, device=dev)
        buf[:R, :C] = t.to(dev)
        return buf[:R, :C]
    ld = ((R + 15) // 16) * 16 + pad
    buf = torch.zeros((max(C, 1), ld), dtype=torch.int8, device=dev)
    buf[:C, :R] = t.t().contiguous().to(dev)
    return buf[:C, :R].t()


def ulp_dist(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    def ordinal(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b)

    return np.abs(ordinal(a_bits) - ordinal(b_bits))


def run_case(M, N, K, la="row", lb="col", out="bf16", stream_k=True, pad=0, vec_scales=True, seed=0):
    rng = np.random.default_rng(seed + M * 31 + N * 7 + K)
    a = synth.weights_np(rng, M, K)
    b = synth.weights_np(rng, K, N)
    sa = synth.scales_np(rng, M)
    sb = synth.scales_np(rng, N)
    dev = torch.device("cuda", 0)
    ta, tb = to_dev(a, la, pad), to_dev(b, lb, pad)
    acc_ref = O.gemm_i8_acc(a, b)
    c32 = api.gemm_quant(ta, tb, out_dtype=torch.int32, stream_k=stream_k)
    torch.cuda.synchronize()
    got = c32.cpu().numpy()
    bad = np.argwhere(got != acc_ref)
    assert bad.size == 0, f"int32 mismatch at {bad[:5].tolist()} ({len(bad)} total)"
    if out == "i32":
        return
    dt = torch.float16 if out == "f16" else torch.bfloat16
    if vec_scales:
        c = api.gemm_quant(ta, tb, torch.from_numpy(sa).to(dev), torch.from_numpy(sb).to(dev), out_dtype=dt,
                           stream_k=stream_k)
        ref = O.dequant(acc_ref, sa, sb, out_dtype=out)
    else:  # tensor-scale mode of the reference (scale_a = scale_b = 1/127, :227)
        c = api.gemm_quant(ta, tb, scale_a=1 / 127, scale_b=1 / 127, out_dtype=dt, stream_k=stream_k)
        ref = O.dequant(acc_ref, None, None, np.float32(1 / 127), np.float32(1 / 127), out_dtype=out)
    torch.cuda.synchronize()
    bits = c.view(torch.int16).cpu().numpy().view(np.uint16)
    assert ulp_dist(bits, ref).max() <= ULP_TOL
    assert np.array_equal(bits, ref)  # stronger: identical fp32 epilogue


LAYOUTS = [("row", "col"), ("row", "row"), ("col", "col"), ("col", "row")]


@pytest.mark.parametrize("la,lb", LAYOUTS)
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (130, 200, 304), (384, 768, 2048), (1, 300, 64)])
def test_layouts_shapes(cuda_device, la, lb, M, N, K):
    run_case(M, N, K, la, lb)


@pytest.mark.parametrize("M,N,K", [(16, 2048, 1024), (64, 4096, 512), (1, 1024, 256), (100, 640, 4096),
                                   (33, 28672, 256)])
def test_skinny_m_swap(cuda_device, M, N, K):
    run_case(M, N, K, "row", "col", out="f16")


@pytest.mark.parametrize("M,N,K", [(1000, 1000, 1000), (129, 257, 1040), (517, 95, 333), (300, 300, 100),
                                   (600, 520, 2000)])
def test_ragged_padded(cuda_device, M, N, K):
    run_case(M, N, K, "row", "col", pad=16)
    run_case(M, N, K, "col", "row", pad=32, out="f16")


# CTA-pair shapes whose last round is partly filled: 4096^2 (256 tiles, 34 in
# the last round), 1280 x 4096 (80 -> 6), 16384 x 3584 (896 -> 8, config 4's
# 8-GPU shard), ragged 2500 x 7900 (310 -> 14, last tile past N), MN-major A.
@pytest.mark.parametrize("M,N,K,la", [(4096, 4096, 512, "row"), (1280, 4096, 1024, "row"),
                                      (16384, 3584, 256, "row"), (2500, 7900, 512, "row"),
                                      (4096, 4096, 256, "col")])
def test_pair_partial_last_round(cuda_device, M, N, K, la):
    run_case(M, N, K, la, "col")


@pytest.mark.parametrize("stream_k", [True, False])
def test_stream_k_equivalence(cuda_device, stream_k):
    # 128 x 8192, swapped: 64 1-CTA tiles of 128 x 128 over 148 SMs, all stream-K
    # (or whole tiles without a workspace); and 100 x 16384 with column-major A
    # (not swapped): 64 tiles of 128 x 256, all stream-K
    assert api.plan(128, 8192, 1024).sk_iters > 0 or not stream_k
    run_case(128, 8192, 1024, stream_k=stream_k)
    run_case(100, 16384, 1024, la="col", stream_k=stream_k)


def test_stream_k_workspace_reuse(cuda_device):
    # repeated calls reuse the same workspace; it must come back zeroed
    for i in range(3):
        run_case(128, 8192, 2048, out="f16", seed=i)


def test_tensor_scale_mode(cuda_device):
    run_case(256, 256, 512, out="f16", vec_scales=False)


def test_k_zero_and_empty(cuda_device):
    dev = cuda_device
    a = torch.zeros((4, 0), dtype=torch.int8, device=dev)
    b = torch.zeros((0, 8), dtype=torch.int8, device=dev)
    c = torch.full((4, 8), 3.0, dtype=torch.bfloat16, device=dev)
    api.gemm_quant(a, b, c=c)
    torch.cuda.synchronize()
    assert torch.all(c == 0)


def test_c1_chain_golden(cuda_device):
    """smoothquant -> GEMM on the CPU-runnable configuration against the fixture."""
    from golden.make_golden import GOLDEN

    g = np.load(GOLDEN)
    dev = cuda_device
    y, rs = api.smoothquant(torch.from_numpy(g["x"]).to(dev), torch.from_numpy(g["smooth"]).to(dev))
    w = torch.from_numpy(g["w_nk"]).to(dev)  # [N, K] K-major -> B = w.t()
    acc = api.gemm_quant(y, w.t(), out_dtype=torch.int32)
    out = api.gemm_quant(y, w.t(), rs, torch.from_numpy(g["sb"]).to(dev), out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), g["acc"])
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), g["out_f16"])


def test_full_size_square_8192(cuda_device):
    """C2: 8192^3, A row-major, B column-major, bf16 out.  Whole int32 result
    checked against cuBLASLt's exact int8 GEMM; sampled rows against the oracle."""
    dev = cuda_device
    n = 8192
    a = synth.torch_int8_uniform((n, n), dev, 11)
    w = synth.torch_int8_uniform((n, n), dev, 12)  # [N, K]
    b = w.t()
    c32 = api.gemm_quant(a, b, out_dtype=torch.int32)
    ref = torch._int_mm(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c32, ref)
    rows = torch.arange(0, n, 509, device=dev)
    acc0 = O.gemm_i8_acc(a[rows].cpu().numpy(), w.cpu().numpy().T)
    assert np.array_equal(c32[rows].cpu().numpy(), acc0)
    sa = synth.torch_scales(n, dev, 13)
    sb = synth.torch_scales(n, dev, 14)
    c = api.gemm_quant(a, b, sa, sb, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ref_bits = O.dequant(acc0, sa[rows].cpu().numpy(), sb.cpu().numpy(), out_dtype="bf16")
    assert np.array_equal(c[rows].view(torch.int16).cpu().numpy().view(np.uint16), ref_bits)


@pytest.mark.parametrize("M", [16, 64])
def test_full_size_decode(cuda_device, M):
    """C3: [M, 8192] x [8192, 28672] (K-major weights), fp16 out, whole output vs oracle."""
    dev = cuda_device
    rng = np.random.default_rng(M)
    a = synth.weights_np(rng, M, 8192)
    w = synth.torch_int8_uniform((28672, 8192), dev, 21)
    sa = synth.scales_np(rng, M)
    sb = synth.torch_scales(28672, dev, 22)
    ta = torch.from_numpy(a).to(dev)
    c32 = api.gemm_quant(ta, w.t(), out_dtype=torch.int32)
    c = api.gemm_quant(ta, w.t(), torch.from_numpy(sa).to(dev), sb, out_dtype=torch.float16)
    torch.cuda.synchronize()
    acc0 = O.gemm_i8_acc(a, w.cpu().numpy().T)
    assert np.array_equal(c32.cpu().numpy(), acc0)
    assert np.array_equal(c.view(torch.int16).cpu().numpy().view(np.uint16),
                          O.dequant(acc0, sa, sb.cpu().numpy(), out_dtype="f16"))


def test_no_device_timeout_flag(cuda_device):
    run_case(256, 512, 1024)
    assert api.last_device_error() == 0


def test_bounded_wait_reports_timeout(cuda_device):
    # a wait nothing satisfies gives up after 2 ms and reports TIMEOUT; the context stays usable
    st = api.debug_bounded_wait(2000)
    assert st == 4  # B2SQ_ERR_TIMEOUT
    run_case(128, 256, 256)


@pytest.mark.parametrize("M,N,K,chunks", [(1000, 512, 256, 3), (4096, 1024, 512, 8), (7, 256, 128, 4),
                                          (3000, 2304, 256, 0), (8192, 8192, 256, 0)])
def test_gemm_from_host_buffers(cuda_device, M, N, K, chunks):
    """gemm_quant_host (pinned host operands and result, chunked and overlapped)
    equals gemm_quant on device tensors, bit for bit, and reuses its buffers."""
    from optimized_rocwmma_samples_b200 import api, synth

    dev = cuda_device
    a = synth.torch_int8_uniform((M, K), dev, 11)
    w = synth.torch_int8_uniform((N, K), dev, 12)
    sa, sb = synth.torch_scales(M, dev, 13), synth.torch_scales(N, dev, 14)
    ref = api.gemm_quant(a, w.t(), sa, sb, out_dtype=torch.bfloat16)
    h = [t.cpu().pin_memory() for t in (a, w, sa, sb)]
    h_c = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    bufs = None
    for _ in range(2):
        h_c.zero_()
        bufs = api.gemm_quant_host(*h, h_c, out_dtype=torch.bfloat16, chunks=chunks, buffers=bufs)
        torch.cuda.synchronize()
        assert torch.equal(h_c, ref.cpu())


def test_host_entry_int32_without_scales(cuda_device):
    """b2sq_gemm_i8_host through the C ABI with int32 output and no scale
    vectors (ragged shape, 2 x 3 blocks): equals b2sq_gemm_i8 on device tensors."""
    import ctypes as C

    from optimized_rocwmma_samples_b200 import _lib, api, synth

    dev = cuda_device
    M, N, K = 300, 520, 272
    a = synth.torch_int8_uniform((M, K), dev, 21)
    w = synth.torch_int8_uniform((N, K), dev, 22)
    ref = api.gemm_quant(a, w.t(), out_dtype=torch.int32)
    h_a, h_w = a.cpu().pin_memory(), w.cpu().pin_memory()
    h_c = torch.zeros((M, N), dtype=torch.int32).pin_memory()
    lib = _lib.load()
    size = C.c_size_t(0)
    assert lib.b2sq_gemm_i8_host_buffer_size(M, N, K, _lib.I32, C.byref(size)) == _lib.B2SQ_OK
    buf = torch.empty((size.value,), dtype=torch.uint8, device=dev)
    for _ in range(2):
        h_c.zero_()
        st = lib.b2sq_gemm_i8_host(M, N, K, h_a.data_ptr(), h_w.data_ptr(), None, None, 1.0, 1.0, h_c.data_ptr(),
                                   _lib.I32, buf.data_ptr(), buf.numel(), 2, 3,
                                   torch.cuda.current_stream().cuda_stream)
        assert st == _lib.B2SQ_OK, lib.b2sq_last_error_message()
        torch.cuda.synchronize()
        assert torch.equal(h_c, ref.cpu())
