"""ctypes binding of libb2sq.so (the C ABI declared in include/b2sq.h).

The library is built in-tree by ``optimized_rocwmma_samples_b200.build``.  If
it is missing, loading raises; there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb2sq.so"

B2SQ_OK = 0
B2SQ_ERR_INVALID_ARG = 1
B2SQ_ERR_UNSUPPORTED = 2
B2SQ_ERR_CUDA = 3
B2SQ_ERR_TIMEOUT = 4

ROW_MAJOR = 0
COL_MAJOR = 1

F16 = 0
BF16 = 1
I32 = 2


class GemmPlan(C.Structure):
    _fields_ = [
        ("swap_ab", C.c_uint32),
        ("tile_m", C.c_uint32),
        ("tile_n", C.c_uint32),
        ("tile_k", C.c_uint32),
        ("stages", C.c_uint32),
        ("tiles_m", C.c_uint32),
        ("tiles_n", C.c_uint32),
        ("k_blocks", C.c_uint32),
        ("ctas", C.c_uint32),
        ("dp_tiles", C.c_uint32),
        ("sk_iters_per_cta_floor", C.c_uint32),
        ("sk_iters", C.c_uint64),
        ("cta_pair", C.c_uint32),
    ]


class B2sqError(RuntimeError):
    """A libb2sq call returned a non-OK status."""

    def __init__(self, status: int, fn: str, msg: str):
        self.status = status
        super().__init__(f"{fn}: status {status} ({msg})")


_u32, _u64, _f32, _vp, _sz, _i = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p, C.c_size_t, C.c_int

# name -> (restype, argtypes)
SIGNATURES = {
    "b2sq_smoothquant": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _f32, _vp]),
    "b2sq_moe_smoothquant": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _f32, _vp, _vp]),
    "b2sq_gemm_i8": (_i, [_u32, _u32, _u32, _vp, _i, _u32, _vp, _i, _u32, _vp, _i, _u32,
                          _vp, _vp, _f32, _f32, _vp, _sz, _vp]),
    "b2sq_gemm_i8_no_alloc": (_i, [_u32, _u32, _u32, _vp, _i, _u32, _vp, _i, _u32, _vp, _i, _u32,
                                   _vp, _vp, _f32, _f32, _vp]),
    "b2sq_smoothquant_gemm_i8": (_i, [_vp, _vp, _f32, _vp, _vp, _u32, _u32, _vp, _i, _u32, _u32, _vp, _i, _u32,
                                      _vp, _f32, _vp, _sz, _vp]),
    "b2sq_gemm_i8_host": (_i, [_u32, _u32, _u32, _vp, _vp, _vp, _vp, _f32, _f32, _vp, _i, _vp, _sz, _u32, _u32,
                               _vp]),
    "b2sq_gemm_i8_host_buffer_size": (_i, [_u32, _u32, _u32, _i, C.POINTER(_sz)]),
    "b2sq_gemm_i8_workspace_size": (_i, [_u32, _u32, _u32, _i, _i, C.POINTER(_sz)]),
    "b2sq_gemm_i8_plan": (_i, [_u32, _u32, _u32, _i, _i, _i, _u32, C.POINTER(GemmPlan)]),
    "b2sq_gemm_i8_allgather": (_i, [_u32, _u32, _u32, _vp, _i, _u32, _vp, _i, _u32, _vp, _u32, _u32, _u32, _i, _u32,
                                    _vp, _vp, _f32, _f32, _vp, C.c_size_t, _vp]),
    "b2sq_gemm_i8_allgather_mc": (_i, [_u32, _u32, _u32, _vp, _i, _u32, _vp, _i, _u32, _vp, _vp, _u32, _i, _u32,
                                       _vp, _vp, _f32, _f32, _vp, C.c_size_t, _vp]),
    "b2sq_ipc_export": (_i, [_vp, _vp, C.POINTER(C.c_uint64)]),
    "b2sq_ipc_open": (_i, [_vp, C.POINTER(C.c_void_p)]),
    "b2sq_ipc_close": (_i, [_vp]),
    "b2sq_topk_softmax": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "b2sq_moe_sorting": (_i, [_vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp]),
    "b2sq_gemm_i8_grouped": (_i, [_u32, _u32, _u32, _u32, _vp, _u32, _vp, _u32, _vp, _i, _u32, _vp, _vp,
                                  _f32, _f32, _vp, _vp, _vp]),
    "b2sq_status_string": (C.c_char_p, [_i]),
    "b2sq_last_error_message": (C.c_char_p, []),
    "b2sq_last_device_error": (_i, [_vp, C.POINTER(_u32)]),
    "b2sq_debug_bounded_wait": (_i, [_u32, _vp]),
    "b2sq_version": (C.c_char_p, []),
}

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Loads libb2sq.so once; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m optimized_rocwmma_samples_b200.build` "
                    "(there is no non-CUDA fallback)")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def check(status: int, fn: str) -> None:
    if status != B2SQ_OK:
        lib = load()
        msg = lib.b2sq_last_error_message().decode() or lib.b2sq_status_string(status).decode()
        raise B2sqError(status, fn, msg)
