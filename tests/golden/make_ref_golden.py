"""Generates tests/golden/ref_pin.npz: outputs of the reference's OWN kernels
(kernel_smoothquant, kernel_moe_smoothquant, kernel_topk_softmax[_large] and
the three sorting kernels, rocwmma_*.cpp) run on the CPU through
oracle/_ref/libref.so, on seeded inputs shaped like BASELINE configs 1, 3 and
5 plus edge cases.  The tests compare the oracle and the CUDA kernels with
these outputs, so parity is pinned to the reference's code, not only to its
restatement.

    make -C oracle/refbuild REF=<reference tree>
    python tests/golden/make_ref_golden.py

The C1 case reuses the inputs stored in c1.npz.  Sorting runs with one host
thread (HIPEMU_THREADS=1), so its scatter order is the one a single wave
order gives; the tests compare each expert's segment as a set.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
OUT = HERE / "ref_pin.npz"

for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def inputs() -> dict:
    """Seeded inputs of every case (the C1 case's come from c1.npz)."""
    from optimized_rocwmma_samples_b200 import synth

    d = {}
    c1 = np.load(HERE / "c1.npz")
    d["sq_c1_x"], d["sq_c1_s"] = c1["x"], c1["smooth"]
    rng = np.random.default_rng(20)
    # config 3 (decode): 16 x 8192, 0.1% outlier channels x30
    d["sq_c3_x"] = synth.activations_np(rng, 16, 8192, 8, 30.0)
    d["sq_c3_s"] = synth.smooth_np(rng, 8192)
    # edge cases: ragged N (scalar tail loop), inf / nan / zero / subnormal rows, fractional qmax
    x = synth.activations_np(rng, 8, 1000, 3, 20.0)
    x[0, 5] = np.inf
    x[1, 7] = np.nan
    x[2, :] = 0
    x[3, :] = np.float16(6e-8)
    x[4, 3] = -np.inf
    x[5, 100] = np.float16(65504.0)
    d["sq_edge_x"], d["sq_edge_s"] = x, synth.smooth_np(rng, 1000)
    d["sq_edge_qmax"] = np.array([100.5], np.float32)
    # config 5 (MoE): 32 tokens x 4096, 8 experts, top-2, two invalid ids
    T, H, E, K = 32, 4096, 8, 2
    d["moe_x"] = synth.activations_np(rng, T, H, 4, 20.0)
    d["moe_s"] = synth.smooth_np(rng, H, E)
    ids = synth.topk_routing_np(rng, T, E, K)
    ids[3, 1] = -1
    ids[5, 0] = E
    d["moe_ids"] = ids
    # router: config 5's 8 experts top-2, the reference driver's 32/5 and 64/5, and > 64 experts
    for name, (t, e, k) in {"r8": (512, 8, 2), "r32": (256, 32, 5), "r64": (256, 64, 5), "r128": (64, 128, 8)}.items():
        d[f"topk_{name}_logits"] = rng.standard_normal((t, e)).astype(np.float16)
        d[f"topk_{name}_k"] = np.array([k], np.int32)
    # sorting: the reference driver's 3328 tokens, 8 experts top-4, unit 32, one invalid id
    ids = synth.topk_routing_np(rng, 3328, 8, 4)
    ids[0, 0] = -1
    d["sort_ids"], d["sort_e"], d["sort_unit"] = ids, np.array([8], np.int32), np.array([32], np.int32)
    return d


def generate(write: bool = True) -> dict:
    import ref

    os.environ["HIPEMU_THREADS"] = "1"
    if not ref.available():
        raise SystemExit("oracle/_ref/libref.so is not built (make -C oracle/refbuild REF=...)")
    d = inputs()
    out = {k: v for k, v in d.items() if not k.startswith("sq_c1_")}  # C1 inputs live in c1.npz
    for case in ("c1", "c3", "edge"):
        q = float(d["sq_edge_qmax"][0]) if case == "edge" else 127.0
        out[f"sq_{case}_y"], out[f"sq_{case}_rs"] = ref.smoothquant(d[f"sq_{case}_x"], d[f"sq_{case}_s"], q)
    out["moe_qy"], out["moe_rs"] = ref.moe_smoothquant(d["moe_x"], d["moe_s"], d["moe_ids"], fill=0)
    for name in ("r8", "r32", "r64", "r128"):
        out[f"topk_{name}_w"], out[f"topk_{name}_i"] = ref.topk_softmax(d[f"topk_{name}_logits"],
                                                                        int(d[f"topk_{name}_k"][0]))
    cnt, start, padded, sid = ref.moe_sorting(d["sort_ids"], int(d["sort_e"][0]), int(d["sort_unit"][0]))
    out.update(sort_count=cnt, sort_start=start, sort_padded=padded, sort_sorted=sid)
    if write:
        np.savez_compressed(OUT, **out)
    return out


def load() -> dict:
    """The fixture with the C1 inputs merged back in."""
    d = dict(np.load(OUT))
    c1 = np.load(HERE / "c1.npz")
    d["sq_c1_x"], d["sq_c1_s"] = c1["x"], c1["smooth"]
    return d


if __name__ == "__main__":
    generate()
    print(OUT, OUT.stat().st_size, "bytes")
