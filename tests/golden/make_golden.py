"""Generates tests/golden/c1.npz: the CPU-runnable configuration (x fp16
[256,1024] with 8 outlier columns x20, smooth U[0.5,2], W int8 [1024,512],
per-channel scales, seed 0) pushed through the oracle.

    python tests/golden/make_golden.py

The reference cannot run here (HIP only) and holds no vectors for this path,
so the fixture pins the oracle's outputs; its smoothquant half is
cross-checked against an independent numpy restatement in tests/test_oracle.py.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
GOLDEN = HERE / "c1.npz"

for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def generate(write: bool = True):
    import oracle as O
    from optimized_rocwmma_samples_b200 import synth

    cfg = synth.C1
    x, s, w_nk, sb = synth.config_inputs_np(cfg)
    y, rs = O.smoothquant(x, s)
    # W is stored K-major [N, K]; the GEMM's B = W^T [K, N] (column-major).
    acc = O.gemm_i8_acc(y, w_nk.T)
    out = O.dequant(acc, rs, sb, out_dtype="f16")
    d = dict(x=x, smooth=s, w_nk=w_nk, sb=sb, y=y, row_scale=rs, acc=acc, out_f16=out)
    if write:
        np.savez_compressed(GOLDEN, **d)
    return d


if __name__ == "__main__":
    generate()
    print(GOLDEN, GOLDEN.stat().st_size, "bytes")
