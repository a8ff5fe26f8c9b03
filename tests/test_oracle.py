"""CPU checks of the oracle: known answers from the reference's own driver
inputs, edge cases, an independent numpy restatement, exact conversions and
the committed golden fixture.  No GPU."""
import numpy as np
import pytest
import torch

import oracle as O
from optimized_rocwmma_samples_b200 import synth


def np_smoothquant(x16, s, qmax=127.0):
    """Independent numpy restatement of rocwmma_smoothquant.cpp:74-121 (fp32)."""
    xs = x16.astype(np.float32) * s.astype(np.float32)[None, :]
    amax = np.max(np.abs(xs), axis=1) if xs.shape[1] else np.zeros(xs.shape[0], np.float32)
    rs = (amax / np.float32(qmax)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(rs > 0, np.float32(1.0) / np.where(rs > 0, rs, 1), 0).astype(np.float32)
    v = (xs * inv[:, None]).astype(np.float32)
    q = np.clip(np.rint(v), -qmax, qmax).astype(np.int8)
    return q, rs


# ----------------------------------------------------------------- known answers
def test_kat_reference_driver_inputs():
    # rocwmma_smoothquant.cpp:140-141: x = 0.5, smooth = 1 for M x N.
    M, N = 7, 4096
    y, rs = O.smoothquant(np.full((M, N), 0.5, np.float16), np.ones(N, np.float32))
    assert np.all(y == 127)
    assert np.all(rs == np.float32(0.5) / np.float32(127.0))


def test_kat_moe_reference_driver_inputs():
    # rocwmma_moe_smoothquant.cpp:152-163: constant x/smooth, distinct random expert ids.
    T, H, E, K = 16, 4096, 8, 2
    rng = np.random.default_rng(42)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    qy, rs = O.moe_smoothquant(np.full((T, H), 0.5, np.float16), np.ones((E, H), np.float32), ids)
    assert np.all(qy == 127) and np.all(rs == np.float32(0.5) / np.float32(127.0))


def test_kat_zero_row():
    x = np.zeros((3, 64), np.float16)
    x[1, 5] = 1.0
    y, rs = O.smoothquant(x, np.ones(64, np.float32))
    assert rs[0] == 0 and rs[2] == 0 and np.all(y[0] == 0) and np.all(y[2] == 0)  # inv = 0 (:98)
    assert y[1, 5] == 127


def test_kat_round_half_even():
    # amax 127 with s = 1 -> row_scale 1, inv 1: x*inv is x itself.
    row = np.array([127, 2.5, 3.5, -2.5, -3.5, 0.5, 1.5, -0.5], np.float16)
    y, rs = O.smoothquant(row[None, :], np.ones(8, np.float32))
    assert rs[0] == 1.0
    assert list(y[0]) == [127, 2, 4, -2, -4, 0, 2, 0]


def test_kat_clamp_and_qmax():
    x = np.array([[4.0, -4.0, 1.0, 2.0]], np.float16)
    y, rs = O.smoothquant(x, np.ones(4, np.float32), qmax=7.0)
    assert rs[0] == np.float32(4.0) / np.float32(7.0)
    assert y[0, 0] == 7 and y[0, 1] == -7  # clamp to +-qmax
    y2, _ = np_smoothquant(x, np.ones(4, np.float32), qmax=7.0)  # 2 * fl(1/fl(4/7)) rounds in fp32
    assert np.array_equal(y, y2)


def test_kat_gemm_all_127():
    K = 1024
    a = np.full((4, K), 127, np.int8)
    b = np.full((K, 3), 127, np.int8)
    assert np.all(O.gemm_i8_acc(a, b) == 16129 * K)


def test_kat_gemm_layouts_agree():
    rng = np.random.default_rng(3)
    a = synth.weights_np(rng, 37, 70)
    b = synth.weights_np(rng, 70, 29)
    ref = a.astype(np.int64) @ b.astype(np.int64)
    for aa in (a, np.asfortranarray(a)):
        for bb in (b, np.asfortranarray(b)):
            assert np.array_equal(O.gemm_i8_acc(aa, bb), ref)


# ------------------------------------------------------------- independent check
@pytest.mark.parametrize("M,N", [(64, 1024), (5, 1000), (3, 7), (2, 0)])
def test_smoothquant_matches_numpy(M, N):
    rng = np.random.default_rng(M * 1000 + N)
    x = synth.activations_np(rng, M, N, min(8, N), 20.0) if N else np.zeros((M, 0), np.float16)
    s = synth.smooth_np(rng, N)
    y, rs = O.smoothquant(x, s)
    y2, rs2 = np_smoothquant(x, s)
    assert np.array_equal(rs.view(np.uint32), rs2.view(np.uint32))
    assert np.array_equal(y, y2)


def test_moe_invalid_ids_and_perm():
    rng = np.random.default_rng(5)
    T, H, E, K = 9, 256, 4, 3
    x = synth.activations_np(rng, T, H, 2, 20.0)
    s = synth.smooth_np(rng, H, E)
    ids = rng.integers(0, E, (T, K)).astype(np.int32)
    ids[2, 1] = -1
    ids[4, 0] = E  # out of range: row left unwritten (rocwmma_moe_smoothquant.cpp:86-87)
    sentinel_q = np.full((T * K, H), 55, np.int8)
    sentinel_r = np.full((T * K,), 9.0, np.float32)
    qy, rs = O.moe_smoothquant(x, s, ids, qy=sentinel_q, row_scale=sentinel_r)
    for t in range(T):
        for k in range(K):
            r = t * K + k
            e = ids[t, k]
            if e < 0 or e >= E:
                assert np.all(qy[r] == 55) and rs[r] == 9.0
            else:
                y1, rs1 = np_smoothquant(x[t:t + 1], s[e])
                assert np.array_equal(qy[r], y1[0]) and rs[r] == rs1[0]
    perm = rng.permutation(T * K).astype(np.int32)
    qp, rp = O.moe_smoothquant(x, s, ids, row_perm=perm)
    valid = (ids.reshape(-1) >= 0) & (ids.reshape(-1) < E)
    assert np.array_equal(qp[perm[valid]], qy[valid])
    assert np.array_equal(rp[perm[valid]], rs[valid])


def test_gemm_matches_int64():
    rng = np.random.default_rng(11)
    a = synth.weights_np(rng, 65, 300)
    b = synth.weights_np(rng, 300, 47)
    assert np.array_equal(O.gemm_i8_acc(a, b), (a.astype(np.int64) @ b.astype(np.int64)).astype(np.int32))


# ------------------------------------------------------------------- conversions
def test_half_to_float_all_values():
    lib = O.load()
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([lib.oracle_half_to_float(int(b)) for b in bits[::7]], np.float32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))


def test_float_to_half_and_bf16_rne():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(1e3),
        rng.standard_normal(2000).astype(np.float32) * np.float32(1e-6),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 5.96e-8, 2.98e-8,
                  1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11, 1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8], np.float32),
    ])
    acc = np.zeros((1, vals.size), np.int32)
    # dequant with acc as float input: use acc=1 and per-column scale = value (1.0 * (1*v) = v exactly)
    acc[:] = 1
    h = O.dequant(acc, None, vals, 1.0, 1.0, "f16")[0]
    assert np.array_equal(h, vals.astype(np.float16).view(np.uint16))
    bf = O.dequant(acc, None, vals, 1.0, 1.0, "bf16")[0]
    ref = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bf, ref)


def test_dequant_order():
    acc = np.array([[123456789, -7]], np.int32)
    sa = np.array([3e-3], np.float32)
    sb = np.array([7e-3, 1e-2], np.float32)
    out = O.dequant(acc, sa, sb, out_dtype="bf16")
    v = (acc.astype(np.float32) * (sa[:, None] * sb[None, :]).astype(np.float32)).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(out, ref)


# ------------------------------------------------------------------------ golden
def test_golden_c1_fixture():
    from golden.make_golden import GOLDEN, generate

    if not GOLDEN.exists():
        pytest.skip("golden fixture not generated")
    g = np.load(GOLDEN)
    x, s, w_nk, sb = synth.config_inputs_np(synth.C1)
    assert np.array_equal(g["x"], x) and np.array_equal(g["w_nk"], w_nk)
    fresh = generate(write=False)
    for k in ("y", "row_scale", "acc", "out_f16"):
        assert np.array_equal(g[k], fresh[k]), k
    # the fixture is also internally consistent with the numpy restatement
    y2, rs2 = np_smoothquant(g["x"], g["smooth"])
    assert np.array_equal(g["y"], y2) and np.array_equal(g["row_scale"], rs2)


def test_kat_moe_sorting():
    # 4 tokens, top-2, 3 experts, unit_size 4; id -1 and 5 are invalid (rocwmma_moe_sorting.cpp:70, :120)
    ids = np.array([[0, 2], [2, 1], [-1, 2], [0, 5]], np.int32)
    cnt, start, sids, perm = O.moe_sorting(ids, 3, 4)
    assert list(cnt) == [2, 1, 3]
    assert list(start) == [0, 4, 8, 12]  # counts padded to 4 (:93-96), sentinel total at [E]
    assert list(sids[:12]) == [0, 3, 4, 4, 1, 4, 4, 4, 0, 1, 2, 4]  # padding slots hold `tokens` (4)
    assert list(perm) == [0, 8, 9, 4, -1, 10, 1, -1]


# ----------------------------------------------------------------- MoE router
def np_topk_softmax(logits16, topk):
    """Independent restatement for well-separated inputs: float64 softmax, stable
    arg-sort (ties to the lower id), as rocwmma_topk_softmax.cpp:58-131 selects."""
    x = logits16.astype(np.float64)
    z = np.exp(x - x.max(axis=1, keepdims=True))
    p = z / z.sum(axis=1, keepdims=True)
    order = np.argsort(-p, axis=1, kind="stable")[:, :topk]
    return np.take_along_axis(p, order, axis=1), order.astype(np.int32)


def test_route_exp_accuracy():
    import math

    rng = np.random.default_rng(5)
    xs = np.concatenate([rng.uniform(-103.9, 88.7, 20000), rng.uniform(-1, 0, 5000)]).astype(np.float32)
    for x in xs:
        t = math.exp(float(x))
        ulp = float(np.spacing(np.float32(t))) if t >= float(np.finfo(np.float32).tiny) else 2.0 ** -149
        assert abs(O.route_exp(float(x)) - t) <= ulp, x
    assert O.route_exp(0.0) == 1.0 and O.route_exp(float("-inf")) == 0.0 and O.route_exp(-200.0) == 0.0
    assert O.route_exp(100.0) == float("inf") and math.isnan(O.route_exp(float("nan")))


@pytest.mark.parametrize("E,K", [(8, 2), (16, 2), (32, 5), (64, 5), (5, 3), (128, 4), (300, 8)])
def test_topk_softmax_matches_float64_restatement(E, K):
    rng = np.random.default_rng(E * 10 + K)
    T = 256
    # distinct logits per row (a permutation of a spread grid): no near-ties
    grid = np.linspace(-4, 4, E).astype(np.float16)
    logits = np.stack([rng.permutation(grid) for _ in range(T)])
    w, i = O.topk_softmax(logits, K)
    w64, i64 = np_topk_softmax(logits, K)
    if E > 64:  # the wide variant only considers experts 0..63 (rocwmma_topk_softmax.cpp:160-164)
        w64, i64 = np_topk_softmax(logits[:, :64], K)
        full = np.exp(logits.astype(np.float64) - logits.astype(np.float64).max(1, keepdims=True))
        w64 = w64 * full[:, :64].sum(1, keepdims=True) / full.sum(1, keepdims=True)
    assert np.array_equal(i, i64)
    assert np.allclose(w, w64, rtol=4e-7, atol=0)


def test_topk_softmax_ties_and_edges():
    # equal logits: equal probabilities; ties resolve in the wave's shfl_down
    # tree order (lane l takes lane l+off only if strictly greater), which after
    # lane 0 is masked reaches lane 4 through offset 4 first: 0, then 4, then 2
    w, i = O.topk_softmax(np.zeros((2, 8), np.float16), 3)
    assert i.tolist() == [[0, 4, 2]] * 2 and np.all(w == np.float32(0.125))
    # topk > experts (<= 64): slots past `experts` untouched
    w, i = O.topk_softmax(np.array([[1.0, 3.0, 2.0]], np.float16), 5, out_w=np.full((1, 5), 7, np.float32),
                          out_i=np.full((1, 5), 9, np.int32))
    assert i.tolist() == [[1, 2, 0, 9, 9]] and w[0, 3] == 7
    # wide variant exhausted: (-1, -1)
    w, i = O.topk_softmax(np.zeros((1, 65), np.float16), 66)
    assert i[0, 64] == -1 and w[0, 65] == -1 and sorted(i[0, :64].tolist()) == list(range(64))
    # all -inf: NaN probabilities; the first lane keeps its NaN (other > NaN is false)
    w, i = O.topk_softmax(np.full((1, 4), -np.inf, np.float16), 2)
    assert np.isnan(w[0, 0]) and i[0, 0] == 0
