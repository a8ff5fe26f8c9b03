"""The CUDA kernels against the reference's own outputs
(tests/golden/ref_pin.npz: the reference's HIP kernels compiled unchanged for
the CPU, see tests/test_ref_pin.py), through the C ABI: smoothquant, MoE
smoothquant, router and sorting, with the same bars as the oracle tests."""
import numpy as np
import pytest
import torch

from optimized_rocwmma_samples_b200 import api
from tests.golden import make_ref_golden as G
from tests.test_ref_pin import ROUTER_ULP, same_f32, ulp_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pin():
    return G.load()


@pytest.mark.parametrize("case", ["c1", "c3", "edge"])
def test_smoothquant_matches_reference(cuda_device, pin, case):
    q = float(pin["sq_edge_qmax"][0]) if case == "edge" else 127.0
    x = torch.from_numpy(pin[f"sq_{case}_x"]).to(cuda_device)
    s = torch.from_numpy(pin[f"sq_{case}_s"]).to(cuda_device)
    y, rs = api.smoothquant(x, s, quant_max=q)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), pin[f"sq_{case}_y"])
    assert same_f32(rs.cpu().numpy(), pin[f"sq_{case}_rs"])


def test_moe_smoothquant_matches_reference(cuda_device, pin):
    dev = cuda_device
    ids = pin["moe_ids"]
    rows = ids.size
    qy = torch.zeros((rows, pin["moe_x"].shape[1]), dtype=torch.int8, device=dev)
    rs = torch.zeros((rows,), dtype=torch.float32, device=dev)
    api.moe_smoothquant(torch.from_numpy(pin["moe_x"]).to(dev), torch.from_numpy(pin["moe_s"]).to(dev),
                        torch.from_numpy(ids).to(dev), qy=qy, row_scale=rs)
    torch.cuda.synchronize()
    assert np.array_equal(qy.cpu().numpy(), pin["moe_qy"])
    assert same_f32(rs.cpu().numpy(), pin["moe_rs"])


@pytest.mark.parametrize("name", ["r8", "r32", "r64", "r128"])
def test_router_matches_reference(cuda_device, pin, name):
    w, i = api.topk_softmax(torch.from_numpy(pin[f"topk_{name}_logits"]).to(cuda_device),
                            int(pin[f"topk_{name}_k"][0]))
    torch.cuda.synchronize()
    assert np.array_equal(i.cpu().numpy(), pin[f"topk_{name}_i"])
    assert ulp_f32(w.cpu().numpy(), pin[f"topk_{name}_w"]).max() <= ROUTER_ULP


def test_sorting_matches_reference(cuda_device, pin):
    E, unit = int(pin["sort_e"][0]), int(pin["sort_unit"][0])
    cnt, start, sid, _ = api.moe_sorting(torch.from_numpy(pin["sort_ids"]).to(cuda_device), E, unit)
    torch.cuda.synchronize()
    cnt, start, sid = cnt.cpu().numpy(), start.cpu().numpy(), sid.cpu().numpy()
    assert np.array_equal(cnt, pin["sort_count"])
    assert np.array_equal(start[:E + 1], pin["sort_start"])
    for e in range(E):
        a = np.sort(sid[start[e]:start[e] + cnt[e]])
        b = np.sort(pin["sort_sorted"][start[e]:start[e] + cnt[e]])
        assert np.array_equal(a, b), f"expert {e}"
