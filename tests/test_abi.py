"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, validates arguments before touching CUDA, and its scheduler covers
every (tile, k-block) exactly once.  No GPU needed."""
import ctypes as C
import re
from pathlib import Path

import pytest

from optimized_rocwmma_samples_b200 import _lib, api

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "b2sq.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"B2SQ_API\s+[\w\s\*]+?\b(b2sq_\w+)\s*\(", text)))


def test_header_symbols_exported():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_version_and_strings():
    lib = _lib.load()
    assert b"sm_100a" in lib.b2sq_version()
    assert lib.b2sq_status_string(0) == b"ok"
    assert lib.b2sq_status_string(4) == b"device wait timed out"


def test_gemm_argument_validation_without_gpu():
    lib = _lib.load()
    ok = lib.b2sq_gemm_i8(0, 16, 16, None, 0, 16, None, 1, 16, None, 1, 16, None, None, 1.0, 1.0, None, 0, None)
    assert ok == _lib.B2SQ_OK  # empty problem: no-op
    buf = (C.c_int8 * 64)()
    addr = C.addressof(buf)
    # bad layout
    assert lib.b2sq_gemm_i8(16, 16, 16, addr, 7, 16, addr, 1, 16, addr, 1, 16, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_INVALID_ARG
    # bad dtype
    assert lib.b2sq_gemm_i8(16, 16, 16, addr, 0, 16, addr, 1, 16, addr, 9, 16, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_INVALID_ARG
    # null output
    assert lib.b2sq_gemm_i8(16, 16, 16, addr, 0, 16, addr, 1, 16, None, 1, 16, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_INVALID_ARG
    # ldc < n
    assert lib.b2sq_gemm_i8(16, 16, 16, addr, 0, 16, addr, 1, 16, addr, 1, 8, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_INVALID_ARG
    # lda < k
    assert lib.b2sq_gemm_i8(16, 16, 32, addr, 0, 16, addr, 1, 32, addr, 1, 16, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_INVALID_ARG
    # lda not a multiple of 16 -> unsupported (TMA)
    aligned = (addr + 15) & ~15
    assert lib.b2sq_gemm_i8(16, 16, 20, aligned, 0, 24, aligned, 1, 32, aligned, 1, 16, None, None, 1, 1, None, 0,
                            None) == _lib.B2SQ_ERR_UNSUPPORTED
    assert b"multiples of 16" in lib.b2sq_last_error_message()
    # misaligned operand -> unsupported
    assert lib.b2sq_gemm_i8(16, 16, 16, aligned + 1, 0, 16, aligned, 1, 16, aligned, 1, 16, None, None, 1, 1,
                            None, 0, None) == _lib.B2SQ_ERR_UNSUPPORTED


def test_smoothquant_argument_validation_without_gpu():
    lib = _lib.load()
    buf = (C.c_float * 16)()
    p = C.addressof(buf)
    assert lib.b2sq_smoothquant(p, p, p, p, 4, 4, 0.0, None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_smoothquant(p, p, p, p, 4, 4, float("nan"), None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_smoothquant(p, p, p, p, 0, 4, 127.0, None) == _lib.B2SQ_OK
    assert lib.b2sq_smoothquant(None, p, p, p, 4, 4, 127.0, None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_moe_smoothquant(p, p, None, p, p, 4, 4, 2, 8, 127.0, None, None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_moe_smoothquant(p, p, p, p, p, 0, 4, 2, 8, 127.0, None, None) == _lib.B2SQ_OK
    assert lib.b2sq_debug_bounded_wait(0, None) == _lib.B2SQ_ERR_INVALID_ARG


def simulate_units(pl):
    """Host restatement of the kernel's per-CTA work list (UnitIter in gemm_i8.cu)."""
    T = pl.tiles_m * pl.tiles_n
    kb = pl.k_blocks
    cover = {}
    workers = pl.ctas // 2 if pl.cta_pair else pl.ctas  # a CTA pair shares one work list
    for cta in range(workers):
        t = cta
        while t < pl.dp_tiles:
            cover.setdefault(t, []).append((0, kb))
            t += workers
        pos = cta * pl.sk_iters // pl.ctas
        end = (cta + 1) * pl.sk_iters // pl.ctas
        while pos < end:
            tt, k0 = divmod(pos, kb)
            k1 = min(kb, k0 + (end - pos))
            cover.setdefault(pl.dp_tiles + tt, []).append((k0, k1))
            pos += k1 - k0
    return T, kb, cover


@pytest.mark.parametrize("m,n,k", [(8192, 8192, 8192), (16, 28672, 8192), (64, 28672, 8192),
                                   (16384, 28672, 8192), (19 * 128, 20 * 256, 1024), (1, 16, 16), (512, 8192, 8192), (200, 8192, 1024), (128, 8192, 8192),
                                   (3000, 3000, 3000), (128, 128, 128 * 1000)])
@pytest.mark.parametrize("sk", [True, False])
def test_schedule_covers_each_kblock_once(m, n, k, sk):
    pl = api.plan(m, n, k, api.ROW_MAJOR, api.COL_MAJOR, use_stream_k=sk, num_sms=148)
    assert pl.ctas <= 148
    T, kb, cover = simulate_units(pl)
    assert set(cover) == set(range(T))
    for t, ranges in cover.items():
        ranges.sort()
        pos = 0
        for k0, k1 in ranges:
            assert k0 == pos and k1 > k0
            pos = k1
        assert pos == kb


def test_plan_choices():
    p = api.plan(16, 28672, 8192, num_sms=148)
    # decode: skinny tiles are HBM-bound, whole tiles only (no stream-K)
    assert p.swap_ab == 1 and p.tile_n == 16 and p.tiles_m == 224 and p.dp_tiles == 224 and p.sk_iters == 0
    p = api.plan(128, 8192, 8192, num_sms=148)
    assert p.swap_ab == 1 and p.tile_n == 128 and p.dp_tiles == 0  # 64 tiles, under a round: all stream-K
    p = api.plan(100, 4096, 4096, num_sms=148)
    assert p.swap_ab == 1 and p.dp_tiles == 32 and p.sk_iters == 0  # 32 tiles: > 3 contributors each, whole tiles
    p = api.plan(96, 28672, 8192, num_sms=148)
    assert p.dp_tiles == 224 and p.sk_iters == 0  # 1.5 rounds: whole tiles
    p = api.plan(8192, 8192, 8192, num_sms=148)
    # CTA pairs: 1024 tiles of 256 x 256 over 74 pairs, 14 rounds, 1.2% idle
    assert p.cta_pair == 1 and p.swap_ab == 0 and p.tile_m == 256 and p.tile_n == 256
    assert p.tiles_m * p.tiles_n == 1024 and p.dp_tiles == 1024 and p.sk_iters == 0 and p.ctas == 148
    p = api.plan(8192, 8192, 8192, api.COL_MAJOR, api.ROW_MAJOR, num_sms=148)  # the reference's layouts: pairs too
    assert p.cta_pair == 1 and p.tile_n == 256 and p.dp_tiles == 1024 and p.sk_iters == 0
    p = api.plan(19 * 128, 20 * 256, 1024, num_sms=148)
    assert p.cta_pair == 1 and p.dp_tiles == 10 * 20  # CTA pairs even with 2.7 rounds (L2-bound 1-CTA tiles lose)
    p = api.plan(512, 8192, 8192, num_sms=148)
    assert p.cta_pair == 1 and p.dp_tiles == 64 and p.ctas == 128  # fewer tiles than pairs: one tile per pair
    p = api.plan(200, 8192, 1024, num_sms=148)
    # more than 128 rows, not skinny enough to swap: CTA pairs (rows past 200 are zero-filled)
    assert p.cta_pair == 1 and p.tiles_m == 1 and p.tiles_n == 32 and p.sk_iters == 0
    p = api.plan(100, 16384, 2048, api.COL_MAJOR, api.COL_MAJOR, num_sms=148)
    # column-major A is not swapped: 1-CTA 128 x 256 tiles, 64 of them, all stream-K
    assert p.cta_pair == 0 and p.tile_n == 256 and p.dp_tiles == 0 and p.sk_iters == 64 * p.k_blocks
    p = api.plan(8192, 8192, 8192, api.ROW_MAJOR, api.ROW_MAJOR, num_sms=148)
    assert p.tile_n in (128, 256)


def test_moe_entry_points_validation_without_gpu():
    lib = _lib.load()
    buf = (C.c_int32 * 64)()
    p = C.addressof(buf)
    assert lib.b2sq_moe_sorting(p, 4, 2, 0, 1, p, p, p, p, None) == _lib.B2SQ_ERR_INVALID_ARG  # no experts
    assert lib.b2sq_moe_sorting(p, 4, 2, 2000, 1, p, p, p, p, None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_moe_sorting(p, 4, 2, 8, 0, p, p, p, p, None) == _lib.B2SQ_ERR_INVALID_ARG  # unit_size 0
    assert lib.b2sq_gemm_i8_grouped(0, 16, 16, 16, p, 16, p, 16, p, 1, 16, None, None, 1, 1, p, p,
                                    None) == _lib.B2SQ_OK  # no groups: no-op
    assert lib.b2sq_gemm_i8_grouped(2, 16, 16, 16, p, 16, p, 16, p, 7, 16, None, None, 1, 1, p, p,
                                    None) == _lib.B2SQ_ERR_INVALID_ARG  # dtype
    assert lib.b2sq_gemm_i8_grouped(2, 16, 16, 16, p, 8, p, 16, p, 1, 16, None, None, 1, 1, p, p,
                                    None) == _lib.B2SQ_ERR_INVALID_ARG  # lda < k
    assert lib.b2sq_gemm_i8_grouped(2, 16, 16, 24, (p + 15) & ~15, 24, (p + 15) & ~15, 32, p, 1, 16, None, None, 1, 1,
                                    p, p, None) == _lib.B2SQ_ERR_UNSUPPORTED  # lda % 16


def test_allgather_and_ipc_validation_without_gpu():
    lib = _lib.load()
    buf = (C.c_int8 * 256)()
    p = (C.addressof(buf) + 15) & ~15
    two = (C.c_void_p * 2)(p, p)
    args = (16, 16, 16, p, 0, 16, p, 1, 16)
    tail = (None, None, 1.0, 1.0, None, 0, None)
    assert lib.b2sq_gemm_i8_allgather(*args, two, 0, 0, 0, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG  # world 0
    assert lib.b2sq_gemm_i8_allgather(*args, two, 9, 0, 0, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG  # world > 8
    assert lib.b2sq_gemm_i8_allgather(*args, two, 2, 2, 0, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG  # rank
    assert lib.b2sq_gemm_i8_allgather(*args, None, 2, 0, 0, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_gemm_i8_allgather(*args, two, 2, 0, 8, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG  # off + n > ldc
    nul = (C.c_void_p * 2)(p, None)
    assert lib.b2sq_gemm_i8_allgather(*args, nul, 2, 0, 0, 1, 16, *tail) == _lib.B2SQ_ERR_INVALID_ARG
    skew = (C.c_void_p * 2)(p, p + 2)  # destinations must share their 16-byte alignment
    assert lib.b2sq_gemm_i8_allgather(*args, skew, 2, 0, 0, 1, 16, *tail) == _lib.B2SQ_ERR_UNSUPPORTED
    h = (C.c_ubyte * 64)()
    off = C.c_uint64(0)
    assert lib.b2sq_ipc_export(None, h, C.byref(off)) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_ipc_open(None, None) == _lib.B2SQ_ERR_INVALID_ARG
    assert lib.b2sq_ipc_close(None) == _lib.B2SQ_ERR_INVALID_ARG


def test_host_gemm_entry_validation_without_gpu():
    """b2sq_gemm_i8_host checks its arguments before any CUDA call."""
    lib = _lib.load()
    size = C.c_size_t(0)
    assert lib.b2sq_gemm_i8_host_buffer_size(8192, 8192, 8192, _lib.BF16, C.byref(size)) == _lib.B2SQ_OK
    # A, B, both scale vectors and C, each rounded up to 256 bytes
    assert size.value >= 8192 * 8192 * 2 + 8192 * 8192 * 2 + 2 * 8192 * 4
    h = (C.c_int8 * 4096)()
    hf = (C.c_float * 64)()
    c = (C.c_uint16 * 4096)()
    big = (C.c_uint8 * 4096)()
    # null output
    assert lib.b2sq_gemm_i8_host(64, 64, 64, h, h, hf, hf, 1.0, 1.0, None, _lib.BF16, big, 4096, 0, 0,
                                 None) == _lib.B2SQ_ERR_INVALID_ARG
    # k not a multiple of 16 (TMA)
    assert lib.b2sq_gemm_i8_host(8, 8, 24, h, h, hf, hf, 1.0, 1.0, c, _lib.BF16, big, 4096, 0, 0,
                                 None) == _lib.B2SQ_ERR_UNSUPPORTED
    # device buffer smaller than b2sq_gemm_i8_host_buffer_size
    assert lib.b2sq_gemm_i8_host(64, 64, 64, h, h, hf, hf, 1.0, 1.0, c, _lib.BF16, big, 16, 0, 0,
                                 None) == _lib.B2SQ_ERR_INVALID_ARG
    assert b"buffer" in lib.b2sq_last_error_message()
    # empty problem: nothing to do
    assert lib.b2sq_gemm_i8_host(0, 64, 64, None, None, None, None, 1.0, 1.0, None, _lib.BF16, None, 0, 0, 0,
                                 None) == _lib.B2SQ_OK
