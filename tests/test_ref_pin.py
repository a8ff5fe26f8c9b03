"""Pins the oracle to the reference's own code, on the CPU.

tests/golden/ref_pin.npz holds outputs of the reference's kernels
(rocwmma_smoothquant.cpp:58-122, rocwmma_moe_smoothquant.cpp:69-131,
rocwmma_topk_softmax.cpp:58-187, rocwmma_moe_sorting.cpp:53-125) compiled
unchanged for the CPU through a HIP host emulation (oracle/refbuild/, made by
tests/golden/make_ref_golden.py).  The oracle must reproduce them:
  * smoothquant and MoE smoothquant: int8 outputs and fp32 row scales bit-exact
    (NaN compared as NaN);
  * router: indices exact, weights within ROUTER_ULP (the reference build's
    expf is the host C library's, the oracle's is its own, both within 1 ulp
    of the exact function, and the softmax sums propagate the difference);
  * sorting: counts and padded starts exact, each expert's segment the same
    set of token ids (the order inside a segment is whatever the reference's
    atomics produce).
Where the reference build itself is present (oracle/_ref/libref.so), a second
set of tests compares the oracle with it live on fresh seeds.  No GPU."""
import numpy as np
import pytest

import oracle as O
import ref
from tests.golden import make_ref_golden as G

ROUTER_ULP = 4


@pytest.fixture(scope="module")
def pin():
    return G.load()


def same_f32(a, b):
    return bool(((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all())


def ulp_f32(a, b):
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))


@pytest.mark.parametrize("case", ["c1", "c3", "edge"])
def test_oracle_smoothquant_matches_reference(pin, case):
    q = float(pin["sq_edge_qmax"][0]) if case == "edge" else 127.0
    y, rs = O.smoothquant(pin[f"sq_{case}_x"], pin[f"sq_{case}_s"], q)
    assert np.array_equal(y, pin[f"sq_{case}_y"])
    assert same_f32(rs, pin[f"sq_{case}_rs"])


def test_oracle_moe_smoothquant_matches_reference(pin):
    qy, rs = O.moe_smoothquant(pin["moe_x"], pin["moe_s"], pin["moe_ids"])
    # rows of invalid expert ids are not written by either (zero-initialised)
    assert np.array_equal(qy, pin["moe_qy"])
    assert same_f32(rs, pin["moe_rs"])


@pytest.mark.parametrize("name", ["r8", "r32", "r64", "r128"])
def test_oracle_router_matches_reference(pin, name):
    w, i = O.topk_softmax(pin[f"topk_{name}_logits"], int(pin[f"topk_{name}_k"][0]))
    assert np.array_equal(i, pin[f"topk_{name}_i"])
    assert ulp_f32(w, pin[f"topk_{name}_w"]).max() <= ROUTER_ULP


def check_sorting(ids, E, unit, cnt, start, sorted_ids):
    c0, st0, sid0, _ = O.moe_sorting(ids, E, unit)
    assert np.array_equal(c0, cnt)
    assert np.array_equal(st0, start)
    for e in range(E):
        a = np.sort(sorted_ids[start[e]:start[e] + cnt[e]])
        b = np.sort(sid0[st0[e]:st0[e] + c0[e]])
        assert np.array_equal(a, b), f"expert {e}"


def test_oracle_sorting_matches_reference(pin):
    check_sorting(pin["sort_ids"], int(pin["sort_e"][0]), int(pin["sort_unit"][0]), pin["sort_count"],
                  pin["sort_start"], pin["sort_sorted"])
    assert np.array_equal(pin["sort_padded"], np.diff(pin["sort_start"]))


def test_reference_known_answer_in_fixture(pin):
    # the reference driver's own known answer holds in the fixture's build too
    # (x = 0.5, s = 1 -> 127 and 0.5/127, rocwmma_smoothquant.cpp:140-141)
    if not ref.available():
        pytest.skip("reference build not present")
    y, rs = ref.smoothquant(np.full((3, 4096), 0.5, np.float16), np.ones(4096, np.float32))
    assert np.all(y == 127) and np.all(rs == np.float32(0.5) / np.float32(127.0))


# ------------------------------------------------------------ live, where built
live = pytest.mark.skipif(not ref.available(), reason="oracle/_ref/libref.so not built (needs the reference tree)")


@live
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_live_smoothquant(seed):
    from optimized_rocwmma_samples_b200 import synth

    rng = np.random.default_rng(seed)
    for m, n, q in [(64, 1024, 127.0), (9, 777, 50.0), (4, 8192, 127.0), (3, 8, 127.0), (2, 20000, 1.5)]:
        x = synth.activations_np(rng, m, n, 3, 25.0)
        x[0, rng.integers(n)] = np.float16(rng.choice([np.inf, -np.inf, np.nan, 65504.0]))
        s = synth.smooth_np(rng, n)
        y, rs = O.smoothquant(x, s, q)
        y1, rs1 = ref.smoothquant(x, s, q)
        assert np.array_equal(y, y1) and same_f32(rs, rs1), (m, n, q)


@live
def test_live_moe_and_router_and_sorting():
    from optimized_rocwmma_samples_b200 import synth

    rng = np.random.default_rng(9)
    T, H, E, K = 40, 2048, 16, 3
    x = synth.activations_np(rng, T, H, 4, 20.0)
    sm = synth.smooth_np(rng, H, E)
    logits = rng.standard_normal((T, E)).astype(np.float16)
    w1, i1 = ref.topk_softmax(logits, K)
    w0, i0 = O.topk_softmax(logits, K)
    assert np.array_equal(i0, i1) and ulp_f32(w0, w1).max() <= ROUTER_ULP
    q1, r1 = ref.moe_smoothquant(x, sm, i1)
    q0, r0 = O.moe_smoothquant(x, sm, i0)
    assert np.array_equal(q0, q1) and same_f32(r0, r1)
    cnt, start, _, sid = ref.moe_sorting(i1, E, 16)
    check_sorting(i1, E, 16, cnt, start, sid)
