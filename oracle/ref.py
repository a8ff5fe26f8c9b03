"""ctypes binding of oracle/_ref/libref.so: the reference's own HIP kernels
(smoothquant, MoE smoothquant, top-k softmax router, MoE sorting) compiled
unchanged for the CPU through the HIP host emulation in oracle/refbuild/.

Test infrastructure only.  It pins the oracle restatement (oracle.c) to the
reference's code: tests/golden/make_ref_golden.py runs these on seeded inputs
and freezes the outputs as fixtures, which the tests compare with the oracle
and the CUDA kernels.  Building needs the reference tree (make -C
oracle/refbuild REF=...); available() is False where it was not built."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libref.so"
_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def load():
    global _lib
    if _lib is None:
        lib = C.CDLL(str(LIB_PATH))
        vp, u32, f32 = C.c_void_p, C.c_uint32, C.c_float
        lib.ref_smoothquant.argtypes = [vp, vp, vp, vp, u32, u32, f32]
        lib.ref_moe_smoothquant.argtypes = [vp, vp, vp, vp, vp, u32, u32, u32, u32, f32]
        lib.ref_topk_softmax.argtypes = [vp, vp, vp, u32, u32, u32]
        lib.ref_moe_sorting.argtypes = [vp, u32, u32, u32, u32, vp, vp, vp, vp, u32]
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data


def smoothquant(x: np.ndarray, smooth: np.ndarray, qmax: float = 127.0):
    """kernel_smoothquant (rocwmma_smoothquant.cpp:58-122) on the CPU."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    smooth = np.ascontiguousarray(smooth, dtype=np.float32)
    M, N = x.shape
    y = np.zeros((M, N), np.int8)
    rs = np.zeros((M,), np.float32)
    load().ref_smoothquant(_p(x), _p(smooth), _p(y), _p(rs), M, N, qmax)
    return y, rs


def moe_smoothquant(x, smooth, topk_ids, qmax: float = 127.0, fill: int = 0):
    """kernel_moe_smoothquant (rocwmma_moe_smoothquant.cpp:69-131); rows of
    invalid expert ids keep `fill` (the kernel does not write them)."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    smooth = np.ascontiguousarray(smooth, dtype=np.float32)
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    T, H = x.shape
    E = smooth.shape[0]
    K = ids.shape[1]
    qy = np.full((T * K, H), fill, np.int8)
    rs = np.full((T * K,), float(fill), np.float32)
    load().ref_moe_smoothquant(_p(x), _p(smooth), _p(ids), _p(qy), _p(rs), T, H, K, E, qmax)
    return qy, rs


def topk_softmax(logits, topk: int):
    """kernel_topk_softmax / _large (rocwmma_topk_softmax.cpp:58-187)."""
    lg = np.ascontiguousarray(logits, dtype=np.float16)
    T, E = lg.shape
    w = np.zeros((T, topk), np.float32)
    i = np.zeros((T, topk), np.int32)
    load().ref_topk_softmax(_p(lg), _p(w), _p(i), T, E, topk)
    return w, i


def moe_sorting(topk_ids, experts: int, unit_size: int):
    """The three sorting kernels (rocwmma_moe_sorting.cpp:53-125) in the
    reference driver's order.  Returns (count [E], start [E+1], padded [E],
    sorted_ids [T*K + E*unit], -1 where nothing was scattered)."""
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    T, K = ids.shape
    n = T * K + experts * unit_size
    cnt = np.zeros(experts, np.int32)
    start = np.zeros(experts + 1, np.int32)
    padded = np.zeros(experts, np.int32)
    sorted_ids = np.zeros(n, np.int32)
    load().ref_moe_sorting(_p(ids), T, K, experts, unit_size, _p(cnt), _p(start), _p(padded), _p(sorted_ids), n)
    return cnt, start, padded, sorted_ids
