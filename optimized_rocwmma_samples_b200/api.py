"""Host-side mirror of the reference operators over the C ABI.

PyTorch supplies device memory and the current stream; every computation is
one call into libb2sq.so.  Names and argument meaning follow the reference:

=========================  ===================================================
this module                reference operator (file:line)
=========================  ===================================================
``smoothquant``            kernel_smoothquant, rocwmma_smoothquant.cpp:58-63
``moe_smoothquant``        kernel_moe_smoothquant, rocwmma_moe_smoothquant.cpp:69-76
``gemm_quant``             gemm_quant_tensor_scale, rocwmma_gemm_quantized.cpp:127-132
                           (+ the per-row x per-column mode of its header, :20/:26)
``topk_softmax``           kernel_topk_softmax(_large), rocwmma_topk_softmax.cpp:58-64, :137-141
``moe_sorting``            kernel_moe_sorting_*, rocwmma_moe_sorting.cpp:53-125
=========================  ===================================================

Errors: the reference exits on a HIP error (CHECK_HIP, common.hpp:33-46) and
prints-and-returns on unsupported GEMM shapes (rocwmma_gemm_quantized.cpp:199-203);
here both raise :class:`B2sqError` carrying the library's status code.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import B2sqError, GemmPlan  # noqa: F401  (re-export)

ROW_MAJOR = _lib.ROW_MAJOR
COL_MAJOR = _lib.COL_MAJOR

_DTYPE_CODE = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.int32: _lib.I32}


def _stream_ptr(stream: Optional[torch.cuda.Stream], device: torch.device) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("libb2sq operators take CUDA tensors (device memory)")
        dev = t.device if dev is None else dev
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def smoothquant(x: torch.Tensor, smooth_scale: torch.Tensor, quant_max: float = 127.0,
                y: Optional[torch.Tensor] = None, row_scale: Optional[torch.Tensor] = None,
                stream: Optional[torch.cuda.Stream] = None):
    """x fp16 [M, N] row-major, smooth_scale fp32 [N] -> (y int8 [M, N], row_scale fp32 [M])."""
    if x.dtype != torch.float16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous fp16 [M, N] tensor")
    M, N = x.shape
    if smooth_scale.dtype != torch.float32 or smooth_scale.numel() != N or not smooth_scale.is_contiguous():
        raise ValueError("smooth_scale must be a contiguous fp32 [N] tensor")
    if y is None:
        y = torch.empty((M, N), dtype=torch.int8, device=x.device)
    if row_scale is None:
        row_scale = torch.empty((M,), dtype=torch.float32, device=x.device)
    dev = _need_cuda(x, smooth_scale, y, row_scale)
    lib = _lib.load()
    st = lib.b2sq_smoothquant(x.data_ptr(), smooth_scale.data_ptr(), y.data_ptr(), row_scale.data_ptr(),
                              M, N, float(quant_max), _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_smoothquant")
    return y, row_scale


def moe_smoothquant(x: torch.Tensor, smooth_scale: torch.Tensor, topk_ids: torch.Tensor,
                    quant_max: float = 127.0, qy: Optional[torch.Tensor] = None,
                    row_scale: Optional[torch.Tensor] = None, row_perm: Optional[torch.Tensor] = None,
                    out_rows: Optional[int] = None, stream: Optional[torch.cuda.Stream] = None):
    """x fp16 [T, H], smooth_scale fp32 [E, H], topk_ids int32 [T, topk]
    -> (qy int8 [rows, H], row_scale fp32 [rows]); rows = T*topk unless given."""
    if x.dtype != torch.float16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous fp16 [tokens, hidden] tensor")
    T, H = x.shape
    if smooth_scale.dtype != torch.float32 or smooth_scale.dim() != 2 or smooth_scale.shape[1] != H:
        raise ValueError("smooth_scale must be fp32 [experts, hidden]")
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2 or topk_ids.shape[0] != T:
        raise ValueError("topk_ids must be int32 [tokens, topk]")
    E, topk = smooth_scale.shape[0], topk_ids.shape[1]
    rows = out_rows if out_rows is not None else T * topk
    if qy is None:
        qy = torch.zeros((rows, H), dtype=torch.int8, device=x.device)
    if row_scale is None:
        row_scale = torch.zeros((rows,), dtype=torch.float32, device=x.device)
    if row_perm is not None and (row_perm.dtype != torch.int32 or row_perm.numel() != T * topk):
        raise ValueError("row_perm must be int32 with tokens*topk entries")
    dev = _need_cuda(x, smooth_scale, topk_ids, qy, row_scale, row_perm)
    lib = _lib.load()
    st = lib.b2sq_moe_smoothquant(x.data_ptr(), smooth_scale.contiguous().data_ptr(),
                                  topk_ids.contiguous().data_ptr(), qy.data_ptr(), row_scale.data_ptr(),
                                  T, H, topk, E, float(quant_max), _ptr(row_perm), _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_moe_smoothquant")
    return qy, row_scale


def _layout_of(t: torch.Tensor, rows: int, cols: int):
    """(layout, ld) of a 2-D view [rows, cols]; row-major if stride(1)==1, col-major if stride(0)==1."""
    if t.dim() != 2 or tuple(t.shape) != (rows, cols):
        raise ValueError(f"expected a [{rows}, {cols}] tensor, got {tuple(t.shape)}")
    s0, s1 = t.stride()
    if s1 == 1 and (rows <= 1 or s0 >= cols):
        return ROW_MAJOR, (s0 if rows > 1 else max(s0, cols))
    if s0 == 1 and (cols <= 1 or s1 >= rows):
        return COL_MAJOR, (s1 if cols > 1 else max(s1, rows))
    raise ValueError("operand must be row-major or column-major (unit stride in one dimension)")


def plan(m: int, n: int, k: int, la: int = ROW_MAJOR, lb: int = COL_MAJOR, use_stream_k: bool = True,
         num_sms: int = 0) -> GemmPlan:
    """The schedule b2sq_gemm_i8 runs for this shape (host only when num_sms > 0)."""
    lib = _lib.load()
    p = GemmPlan()
    _lib.check(lib.b2sq_gemm_i8_plan(m, n, k, la, lb, int(use_stream_k), num_sms, C.byref(p)),
               "b2sq_gemm_i8_plan")
    return p


class Workspace:
    """Zero-filled, reusable stream-K workspace (one per device), grown on demand.

    The library leaves it zero-filled after every completed call, so it is
    cleared only when (re)allocated.  Calls sharing it must be stream-ordered.
    """

    def __init__(self):
        self._bufs: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
        if nbytes == 0:
            return None
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(((nbytes + 255) // 256) * 256, dtype=torch.uint8, device=device)
            self._bufs[idx] = buf
        return buf


_default_ws = Workspace()


def workspace_size(m: int, n: int, k: int, la: int = ROW_MAJOR, lb: int = COL_MAJOR) -> int:
    lib = _lib.load()
    out = C.c_size_t(0)
    _lib.check(lib.b2sq_gemm_i8_workspace_size(m, n, k, la, lb, C.byref(out)), "b2sq_gemm_i8_workspace_size")
    return out.value


def gemm_quant(a: torch.Tensor, b: torch.Tensor, scale_a_row: Optional[torch.Tensor] = None,
               scale_b_col: Optional[torch.Tensor] = None, scale_a: float = 1.0, scale_b: float = 1.0,
               out_dtype: torch.dtype = torch.bfloat16, c: Optional[torch.Tensor] = None,
               stream_k: bool = True, workspace: Optional[Workspace] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """c[M,N] = cvt(float(a[M,K] @ b[K,N]) * (sa[m] * sb[n])), int8 operands, int32 accumulation.

    a: int8 [M, K] row- or column-major; b: int8 [K, N] column-major (K-major
    weights, ``w.t()`` of a contiguous [N, K]) or row-major.  out_dtype
    float16 / bfloat16 / int32 (raw accumulators).
    """
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise ValueError("a and b must be int8")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch: a {tuple(a.shape)} b {tuple(b.shape)}")
    M, K = a.shape
    N = b.shape[1]
    la, lda = _layout_of(a, M, K)
    lb, ldb = _layout_of(b, K, N)
    if out_dtype not in _DTYPE_CODE:
        raise ValueError("out_dtype must be float16, bfloat16 or int32")
    if c is None:
        c = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if c.dtype != out_dtype or c.dim() != 2 or tuple(c.shape) != (M, N) or c.stride(1) != 1:
        raise ValueError("c must be a row-major [M, N] tensor of out_dtype")
    for s, nm, L in ((scale_a_row, "scale_a_row", M), (scale_b_col, "scale_b_col", N)):
        if s is not None and (s.dtype != torch.float32 or s.numel() != L or not s.is_contiguous()):
            raise ValueError(f"{nm} must be a contiguous fp32 vector of {L}")
    dev = _need_cuda(a, b, c, scale_a_row, scale_b_col)
    ws, ws_bytes = None, 0
    if stream_k:
        need = workspace_size(M, N, K, la, lb)
        ws = (workspace or _default_ws).get(dev, need)
        ws_bytes = 0 if ws is None else ws.numel()
    lib = _lib.load()
    st = lib.b2sq_gemm_i8(M, N, K, a.data_ptr(), la, lda, b.data_ptr(), lb, ldb, c.data_ptr(),
                          _DTYPE_CODE[out_dtype], c.stride(0) if M > 1 else N, _ptr(scale_a_row),
                          _ptr(scale_b_col), float(scale_a), float(scale_b), _ptr(ws), ws_bytes,
                          _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_gemm_i8")
    return c


def last_device_error(stream: Optional[torch.cuda.Stream] = None) -> int:
    """Reads/clears the device status word; returns the wait-site code (0 = none)."""
    lib = _lib.load()
    where = C.c_uint32(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    lib.b2sq_last_device_error(_stream_ptr(stream, dev), C.byref(where))
    return where.value


def debug_bounded_wait(timeout_us: int, stream: Optional[torch.cuda.Stream] = None) -> int:
    """Runs the bounded-wait self test; returns the library status (TIMEOUT expected)."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    return lib.b2sq_debug_bounded_wait(timeout_us, _stream_ptr(stream, dev))


# Reference operator names.
kernel_smoothquant = smoothquant
kernel_moe_smoothquant = moe_smoothquant
gemm_quant_tensor_scale = gemm_quant


# ----------------------------------------------------------------------------- MoE
class HostGemmBuffers:
    """The two device buffers gemm_quant_host alternates between (one pair per
    shape, dtype and device): consecutive calls use different buffers, so the
    next call's inputs go up while the previous call's result comes down."""

    def __init__(self, m: int, n: int, k: int, out_dtype: torch.dtype, device: torch.device):
        self.key = (m, n, k, out_dtype, device)
        lib = _lib.load()
        size = C.c_size_t(0)
        _lib.check(lib.b2sq_gemm_i8_host_buffer_size(m, n, k, _DTYPE_CODE[out_dtype], C.byref(size)),
                   "b2sq_gemm_i8_host_buffer_size")
        self.bufs = [torch.empty((size.value,), dtype=torch.uint8, device=device) for _ in range(2)]
        self.turn = 0

    def next(self) -> torch.Tensor:
        buf = self.bufs[self.turn]
        self.turn ^= 1
        return buf


def gemm_quant_host(h_a: torch.Tensor, h_w_nk: torch.Tensor, h_sa: torch.Tensor, h_sb: torch.Tensor,
                    h_c: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16, chunks: int = 0,
                    buffers: Optional[HostGemmBuffers] = None, workspace: Optional[Workspace] = None,
                    device: Optional[torch.device] = None, col_chunks: Optional[int] = None) -> HostGemmBuffers:
    """h_c = dequant(h_a @ h_w_nk.T) for operands and result in (pinned) host
    memory, through b2sq_gemm_i8_host: the problem is cut into chunks x
    col_chunks output blocks (0 = the library's choice) whose host->device
    copies, GEMMs and device->host copies overlap.  On return the work is
    queued on the current stream (synchronise it before reading h_c).
    Returns the device buffer holder, to pass back in on the next call.
    `workspace` is accepted for compatibility and unused (the block GEMMs need
    none)."""
    del workspace
    for t, dt in ((h_a, torch.int8), (h_w_nk, torch.int8), (h_sa, torch.float32), (h_sb, torch.float32),
                  (h_c, out_dtype)):
        if t.device.type != "cpu" or t.dtype != dt or not t.is_contiguous():
            raise ValueError("host operands: contiguous CPU tensors of the documented dtypes expected")
    M, K = h_a.shape
    N = h_w_nk.shape[0]
    if h_w_nk.shape[1] != K or h_c.shape != (M, N) or h_sa.numel() != M or h_sb.numel() != N:
        raise ValueError("shape mismatch among the host operands")
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = (M, N, K, out_dtype, dev)
    b = buffers if buffers is not None and buffers.key == key else HostGemmBuffers(M, N, K, out_dtype, dev)
    lib = _lib.load()
    buf = b.next()
    st = lib.b2sq_gemm_i8_host(M, N, K, h_a.data_ptr(), h_w_nk.data_ptr(), h_sa.data_ptr(), h_sb.data_ptr(), 1.0,
                               1.0, h_c.data_ptr(), _DTYPE_CODE[out_dtype], buf.data_ptr(), buf.numel(),
                               int(chunks), int(chunks if col_chunks is None else col_chunks),
                               _stream_ptr(None, dev))
    _lib.check(st, "b2sq_gemm_i8_host")
    return b


def gemm_allgather(a: torch.Tensor, b: torch.Tensor, c_ranks: list, rank: int, col_offset: int, ldc: int,
                   scale_a_row: Optional[torch.Tensor] = None, scale_b_col: Optional[torch.Tensor] = None,
                   scale_a: float = 1.0, scale_b: float = 1.0, out_dtype: torch.dtype = torch.bfloat16,
                   workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None) -> None:
    """This rank's N shard of a column-parallel GEMM, stored into every rank's
    full output buffer (b2sq_gemm_i8_allgather).  c_ranks: device addresses
    (ints) of each rank's row-major [M, ldc] buffer, mapped into this process;
    the shard lands at columns [col_offset, col_offset + N) of all of them."""
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("a int8 [M, K] and b int8 [K, N] expected")
    M, K = a.shape
    N = b.shape[1]
    la, lda = _layout_of(a, M, K)
    lb, ldb = _layout_of(b, K, N)
    if out_dtype not in _DTYPE_CODE:
        raise ValueError("out_dtype must be float16, bfloat16 or int32")
    dev = _need_cuda(a, b, scale_a_row, scale_b_col)
    need = workspace_size(M, N, K, la, lb)
    ws = (workspace or _default_ws).get(dev, need)
    ptrs = (C.c_void_p * len(c_ranks))(*[int(p) for p in c_ranks])
    lib = _lib.load()
    st = lib.b2sq_gemm_i8_allgather(M, N, K, a.data_ptr(), la, lda, b.data_ptr(), lb, ldb, ptrs, len(c_ranks), rank,
                                    col_offset, _DTYPE_CODE[out_dtype], ldc, _ptr(scale_a_row), _ptr(scale_b_col),
                                    float(scale_a), float(scale_b), _ptr(ws), 0 if ws is None else ws.numel(),
                                    _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_gemm_i8_allgather")


def gemm_allgather_mc(a: torch.Tensor, b: torch.Tensor, c_local: int, c_multicast: int, col_offset: int, ldc: int,
                      scale_a_row: Optional[torch.Tensor] = None, scale_b_col: Optional[torch.Tensor] = None,
                      scale_a: float = 1.0, scale_b: float = 1.0, out_dtype: torch.dtype = torch.bfloat16,
                      workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None) -> None:
    """gemm_allgather through an NVSwitch multicast mapping (b2sq_gemm_i8_allgather_mc):
    c_local / c_multicast are the addresses of this rank's [M, ldc] buffer and
    of its multicast view; each output piece is stored once for all ranks."""
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("a int8 [M, K] and b int8 [K, N] expected")
    M, K = a.shape
    N = b.shape[1]
    la, lda = _layout_of(a, M, K)
    lb, ldb = _layout_of(b, K, N)
    dev = _need_cuda(a, b, scale_a_row, scale_b_col)
    ws = (workspace or _default_ws).get(dev, workspace_size(M, N, K, la, lb))
    lib = _lib.load()
    st = lib.b2sq_gemm_i8_allgather_mc(M, N, K, a.data_ptr(), la, lda, b.data_ptr(), lb, ldb, c_local, c_multicast,
                                       col_offset, _DTYPE_CODE[out_dtype], ldc, _ptr(scale_a_row), _ptr(scale_b_col),
                                       float(scale_a), float(scale_b), _ptr(ws), 0 if ws is None else ws.numel(),
                                       _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_gemm_i8_allgather_mc")


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding t, byte offset of t in it)."""
    _need_cuda(t)
    h = (C.c_ubyte * 64)()
    off = C.c_uint64(0)
    _lib.check(_lib.load().b2sq_ipc_export(t.data_ptr(), h, C.byref(off)), "b2sq_ipc_export")
    return bytes(h), int(off.value)


def ipc_open(handle: bytes) -> int:
    """Maps a peer's exported allocation into this process; returns its base address."""
    h = (C.c_ubyte * 64).from_buffer_copy(handle)
    base = C.c_void_p(0)
    _lib.check(_lib.load().b2sq_ipc_open(h, C.byref(base)), "b2sq_ipc_open")
    return int(base.value)


def ipc_close(base: int) -> None:
    _lib.check(_lib.load().b2sq_ipc_close(C.c_void_p(base)), "b2sq_ipc_close")


def topk_softmax(logits: torch.Tensor, topk: int, topk_weights: Optional[torch.Tensor] = None,
                 topk_indices: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None):
    """MoE router (rocwmma_topk_softmax.cpp): softmax over fp16 logits
    [tokens, experts], then the top-k experts per token.

    Returns (topk_weights fp32 [tokens, topk], topk_indices int32 [tokens, topk]).
    With experts <= 64 and topk > experts the slots past `experts` are left as
    they were (zeros when the outputs are allocated here)."""
    if logits.dtype != torch.float16 or logits.dim() != 2 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous fp16 [tokens, experts] tensor")
    T, E = logits.shape
    dev = _need_cuda(logits, topk_weights, topk_indices)
    if topk_weights is None:
        topk_weights = torch.zeros((T, topk), dtype=torch.float32, device=dev)
    if topk_indices is None:
        topk_indices = torch.zeros((T, topk), dtype=torch.int32, device=dev)
    if (topk_weights.shape != (T, topk) or topk_indices.shape != (T, topk) or topk_weights.dtype != torch.float32
            or topk_indices.dtype != torch.int32 or not topk_weights.is_contiguous()
            or not topk_indices.is_contiguous()):
        raise ValueError("topk_weights / topk_indices must be contiguous fp32 / int32 [tokens, topk]")
    lib = _lib.load()
    st = lib.b2sq_topk_softmax(logits.data_ptr(), topk_weights.data_ptr(), topk_indices.data_ptr(), T, E, topk,
                               _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_topk_softmax")
    return topk_weights, topk_indices


def moe_sorting(topk_ids: torch.Tensor, experts: int, unit_size: int = 1,
                stream: Optional[torch.cuda.Stream] = None):
    """Groups (token, slot) pairs by expert (rocwmma_moe_sorting.cpp).

    Returns (expert_count [E], expert_start [E+1], sorted_token_ids
    [tokens*topk + E*unit_size], row_perm [tokens*topk]), all int32 on the device.
    """
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2 or not topk_ids.is_contiguous():
        raise ValueError("topk_ids must be a contiguous int32 [tokens, topk] tensor")
    T, K = topk_ids.shape
    dev = _need_cuda(topk_ids)
    count = torch.empty((experts,), dtype=torch.int32, device=dev)
    start = torch.empty((experts + 1,), dtype=torch.int32, device=dev)
    sorted_ids = torch.empty((T * K + experts * unit_size,), dtype=torch.int32, device=dev)
    row_perm = torch.empty((T * K,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    st = lib.b2sq_moe_sorting(topk_ids.data_ptr(), T, K, experts, unit_size, count.data_ptr(), start.data_ptr(),
                              sorted_ids.data_ptr(), row_perm.data_ptr(), _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_moe_sorting")
    return count, start, sorted_ids, row_perm


def gemm_grouped(a: torch.Tensor, w: torch.Tensor, group_start: torch.Tensor, group_count: torch.Tensor,
                 scale_a_row: Optional[torch.Tensor] = None, scale_b_col: Optional[torch.Tensor] = None,
                 scale_a: float = 1.0, scale_b: float = 1.0, out_dtype: torch.dtype = torch.bfloat16,
                 c: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Per-expert GEMM over expert-sorted rows: a int8 [rows, K] row-major,
    w int8 [E, N, K] (K-major weights), group_start/group_count int32 [>=E].
    Rows outside every group are left untouched in c."""
    if a.dtype != torch.int8 or w.dtype != torch.int8 or a.dim() != 2 or w.dim() != 3:
        raise ValueError("a must be int8 [rows, K], w int8 [E, N, K]")
    rows, K = a.shape
    E, N, K2 = w.shape
    if K2 != K or a.stride(1) != 1 or w.stride(2) != 1 or w.stride(0) != w.stride(1) * N:
        raise ValueError("shape/layout mismatch between a and w")
    if c is None:
        c = torch.zeros((rows, N), dtype=out_dtype, device=a.device)
    dev = _need_cuda(a, w, c, group_start, group_count, scale_a_row, scale_b_col)
    lib = _lib.load()
    st = lib.b2sq_gemm_i8_grouped(E, rows, N, K, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(1),
                                  c.data_ptr(), _DTYPE_CODE[out_dtype], c.stride(0), _ptr(scale_a_row),
                                  _ptr(scale_b_col), float(scale_a), float(scale_b), group_start.data_ptr(),
                                  group_count.data_ptr(), _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_gemm_i8_grouped")
    return c


def smoothquant_gemm(x: torch.Tensor, smooth_scale: torch.Tensor, w_nk: torch.Tensor,
                     scale_w_col: Optional[torch.Tensor] = None, scale_w: float = 1.0, quant_max: float = 127.0,
                     out_dtype: torch.dtype = torch.float16, xq: Optional[torch.Tensor] = None,
                     row_scale: Optional[torch.Tensor] = None, c: Optional[torch.Tensor] = None,
                     workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None):
    """Smoothquant of x [M, K] followed by the int8 GEMM with K-major weights
    w_nk [N, K], in one C-ABI call (the GEMM is launched with programmatic
    dependent launch).  Returns (c, xq, row_scale)."""
    if x.dtype != torch.float16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous fp16 [M, K] tensor")
    M, K = x.shape
    if w_nk.dtype != torch.int8 or w_nk.dim() != 2 or w_nk.shape[1] != K or w_nk.stride(1) != 1:
        raise ValueError("w_nk must be int8 [N, K] with unit stride along K")
    N = w_nk.shape[0]
    xq = torch.empty((M, K), dtype=torch.int8, device=x.device) if xq is None else xq
    row_scale = torch.empty((M,), dtype=torch.float32, device=x.device) if row_scale is None else row_scale
    c = torch.empty((M, N), dtype=out_dtype, device=x.device) if c is None else c
    dev = _need_cuda(x, smooth_scale, w_nk, xq, row_scale, c, scale_w_col)
    need = workspace_size(M, N, K, ROW_MAJOR, COL_MAJOR)
    ws = (workspace or _default_ws).get(dev, need)
    lib = _lib.load()
    st = lib.b2sq_smoothquant_gemm_i8(x.data_ptr(), smooth_scale.data_ptr(), float(quant_max), xq.data_ptr(),
                                      row_scale.data_ptr(), M, K, w_nk.data_ptr(), COL_MAJOR, w_nk.stride(0), N,
                                      c.data_ptr(), _DTYPE_CODE[out_dtype], c.stride(0), _ptr(scale_w_col),
                                      float(scale_w), _ptr(ws), 0 if ws is None else ws.numel(),
                                      _stream_ptr(stream, dev))
    _lib.check(st, "b2sq_smoothquant_gemm_i8")
    return c, xq, row_scale


kernel_topk_softmax = topk_softmax
