"""numpy/ctypes front end of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / reference arm.  The product
(libb2sq.so and the optimized_rocwmma_samples_b200 package) never imports it.

Each function restates a reference operator on the CPU (see oracle.c for the
file:line each one follows).  Parity status: smoothquant is pinned by the
reference driver's own inputs (x = 0.5, s = 1 -> y = 127, row_scale =
0.5f/127); the GEMM is pinned only by exact integer arithmetic (the reference
holds no int8 GEMM vector).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
            build()
        lib = C.CDLL(str(LIB_PATH))
        vp, u32, f32, i = C.c_void_p, C.c_uint32, C.c_float, C.c_int
        lib.oracle_smoothquant.argtypes = [vp, vp, vp, vp, u32, u32, f32]
        lib.oracle_moe_smoothquant.argtypes = [vp, vp, vp, vp, vp, u32, u32, u32, u32, f32, vp]
        lib.oracle_gemm_i8_acc.argtypes = [u32, u32, u32, vp, i, u32, vp, i, u32, vp, u32]
        lib.oracle_dequant.argtypes = [u32, u32, vp, u32, vp, vp, f32, f32, vp, i, u32]
        lib.oracle_half_to_float.argtypes = [C.c_uint16]
        lib.oracle_half_to_float.restype = f32
        lib.oracle_float_to_half.argtypes = [f32]
        lib.oracle_float_to_half.restype = C.c_uint16
        lib.oracle_float_to_bf16.argtypes = [f32]
        lib.oracle_float_to_bf16.restype = C.c_uint16
        lib.oracle_num_threads.restype = i
        lib.oracle_set_num_threads.argtypes = [i]
        lib.oracle_topk_softmax.argtypes = [vp, vp, vp, u32, u32, u32]
        lib.oracle_route_exp.argtypes = [f32]
        lib.oracle_route_exp.restype = f32
        _lib = lib
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def num_threads() -> int:
    return load().oracle_num_threads()


def set_num_threads(n: int) -> None:
    """Thread count of the oracle's parallel loops started from this thread."""
    load().oracle_set_num_threads(int(n))


def smoothquant(x: np.ndarray, smooth: np.ndarray, qmax: float = 127.0):
    """x float16 [M,N], smooth float32 [N] -> (y int8 [M,N], row_scale float32 [M])."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    smooth = np.ascontiguousarray(smooth, dtype=np.float32)
    M, N = x.shape
    y = np.zeros((M, N), np.int8)
    rs = np.zeros((M,), np.float32)
    load().oracle_smoothquant(_p(x), _p(smooth), _p(y), _p(rs), M, N, qmax)
    return y, rs


def moe_smoothquant(x, smooth, topk_ids, qmax: float = 127.0, row_perm=None, out_rows=None,
                    qy=None, row_scale=None):
    """Rows never written (invalid expert id) keep the initial contents of qy/row_scale."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    smooth = np.ascontiguousarray(smooth, dtype=np.float32)
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    T, H = x.shape
    E = smooth.shape[0]
    topk = ids.shape[1]
    rows = out_rows if out_rows is not None else T * topk
    qy = np.zeros((rows, H), np.int8) if qy is None else np.ascontiguousarray(qy, dtype=np.int8).copy()
    rs = np.zeros((rows,), np.float32) if row_scale is None else np.ascontiguousarray(row_scale, np.float32).copy()
    perm = None if row_perm is None else np.ascontiguousarray(row_perm, dtype=np.int32)
    load().oracle_moe_smoothquant(_p(x), _p(smooth), _p(ids), _p(qy), _p(rs), T, H, topk, E, qmax, _p(perm))
    return qy, rs


def gemm_i8_acc(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact int32 a[M,K] @ b[K,N]; numpy arrays in any memory order (C or F)."""
    assert a.dtype == np.int8 and b.dtype == np.int8
    M, K = a.shape
    K2, N = b.shape
    assert K == K2

    def lay(t):
        if t.flags.c_contiguous:
            return 0, t.shape[1], t
        if t.flags.f_contiguous:
            return 1, t.shape[0], t
        t = np.ascontiguousarray(t)
        return 0, t.shape[1], t

    la, lda, a = lay(a)
    lb, ldb, b = lay(b)
    acc = np.zeros((M, N), np.int32)
    load().oracle_gemm_i8_acc(M, N, K, _p(a), la, max(lda, 1), _p(b), lb, max(ldb, 1), _p(acc), N)
    return acc


def dequant(acc: np.ndarray, sa_row=None, sb_col=None, scale_a: float = 1.0, scale_b: float = 1.0,
            out_dtype: str = "bf16") -> np.ndarray:
    """uint16 bit patterns of the fp16/bf16 epilogue output."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    M, N = acc.shape
    sa = None if sa_row is None else np.ascontiguousarray(sa_row, np.float32)
    sb = None if sb_col is None else np.ascontiguousarray(sb_col, np.float32)
    out = np.zeros((M, N), np.uint16)
    load().oracle_dequant(M, N, _p(acc), N, _p(sa), _p(sb), scale_a, scale_b, _p(out),
                          0 if out_dtype == "f16" else 1, N)
    return out


def gemm_quant(a, b, sa_row=None, sb_col=None, scale_a=1.0, scale_b=1.0, out_dtype="bf16"):
    """(acc int32, out uint16 bits) of the full reference-style quantized GEMM."""
    acc = gemm_i8_acc(a, b)
    return acc, dequant(acc, sa_row, sb_col, scale_a, scale_b, out_dtype)


def topk_softmax(logits: np.ndarray, topk: int, out_w=None, out_i=None):
    """rocwmma_topk_softmax.cpp:58-187 restated (oracle.c: oracle_topk_softmax).
    logits fp16 [tokens, experts]; returns (weights fp32, indices int32), each
    [tokens, topk], starting from out_w / out_i (zeros) for unwritten slots."""
    x = np.ascontiguousarray(logits, dtype=np.float16)
    T, E = x.shape
    w = np.zeros((T, topk), np.float32) if out_w is None else out_w.copy()
    i = np.zeros((T, topk), np.int32) if out_i is None else out_i.copy()
    if T and E and topk:
        load().oracle_topk_softmax(_p(x), _p(w), _p(i), T, E, topk)
    return w, i


def route_exp(a: float) -> float:
    return load().oracle_route_exp(a)


def moe_sorting(topk_ids, experts: int, unit_size: int = 1):
    """rocwmma_moe_sorting.cpp:53-125 restated: histogram of valid expert ids,
    exclusive prefix of counts padded to unit_size, scatter of token ids into
    each expert's segment.  The reference's scatter order inside a segment is
    whatever its atomics produce; this restatement uses the stable order
    (increasing flat index).  Padding slots hold the sentinel `tokens`."""
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    T, K = ids.shape
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < experts)
    count = np.bincount(flat[valid], minlength=experts).astype(np.int32)
    padded = ((count + unit_size - 1) // unit_size) * unit_size
    start = np.zeros(experts + 1, np.int32)
    start[1:] = np.cumsum(padded)
    sorted_ids = np.full(T * K + experts * unit_size, T, np.int32)
    row_perm = np.full(T * K, -1, np.int32)
    nxt = start[:-1].copy()
    for f in range(T * K):
        e = flat[f]
        if 0 <= e < experts:
            sorted_ids[nxt[e]] = f // K
            row_perm[f] = nxt[e]
            nxt[e] += 1
    return count, start, sorted_ids, row_perm


def gemm_grouped(a, w, start, count, sa_row=None, sb_col=None, out_dtype="bf16"):
    """Per-group restatement: rows [start[g], start[g]+count[g]) of a times
    w[g] ([N, K] K-major).  Returns (acc int32 [rows, N], out uint16 bits);
    rows outside every group are zero."""
    rows, K = a.shape
    E, N, _ = w.shape
    acc = np.zeros((rows, N), np.int32)
    out = np.zeros((rows, N), np.uint16)
    for g in range(E):
        r0, n = int(start[g]), int(count[g])
        if n == 0:
            continue
        ag = np.ascontiguousarray(a[r0:r0 + n])
        acc_g = gemm_i8_acc(ag, w[g].T)
        acc[r0:r0 + n] = acc_g
        sa = None if sa_row is None else sa_row[r0:r0 + n]
        sb = None if sb_col is None else sb_col[g * N:(g + 1) * N]
        out[r0:r0 + n] = dequant(acc_g, sa, sb, out_dtype=out_dtype)
    return acc, out
