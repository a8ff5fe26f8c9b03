"""The C++ sample driver (reference-style output lines) runs on the GPU, its
known-answer checks pass, and its lines parse the way the reference's
benchmark.sh parses them (benchmark.sh:177-188: '[Tag] ... X ms Y GB/s|TFlops/s')."""
import re
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

BIN = Path(__file__).resolve().parent.parent / "optimized_rocwmma_samples_b200" / "b2sq_samples"
LINE = re.compile(r"^\[(?P<tag>[\w -]+)\] .*?\s+(?P<ms>[0-9.e+-]+) ms(\s+(?P<val>[0-9.e+-]+) (?P<unit>GB/s|TFlops/s))?$")


def test_samples_driver(cuda_device):
    assert BIN.exists(), "build the package first (python -m optimized_rocwmma_samples_b200.build)"
    res = subprocess.run([str(BIN), "all"], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    tags = {}
    for ln in res.stdout.splitlines():
        m = LINE.match(ln.strip())
        if m:
            tags.setdefault(m["tag"], []).append(float(m["ms"]))
    assert len(tags.get("SmoothQuant", [])) == 4
    assert len(tags.get("MoE-SmoothQuant", [])) == 3
    assert len(tags.get("QuantGEMM-I8", [])) == 3
    assert len(tags.get("QuantGEMM-I8-host", [])) == 1
    assert len(tags.get("MoE Sorting", [])) == 5
    assert len(tags.get("TopK-Softmax", [])) == 5
    assert "FAILED" not in res.stdout
