"""Benchmark of the smoothquant -> int8 GEMM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: int8 GEMM M = N = K = 8192, A row-major,
B column-major (K-major weights), per-row x per-column fp32 dequant, bf16 out.
One step = one b2sq_gemm_i8 call.  ``value`` is whole-job TOPS (2*M*N*K per
step per rank) with inputs resident in HBM; L2 (126 MB) is flushed before
every timed step, outside the timed events, by reading a 512 MB buffer (a
read leaves no dirty lines whose write-back would land in the timed kernel).
At N > 1 GPUs the GEMM is N-sharded (column-parallel weights, weak scaling:
every rank owns an 8192-column weight shard and the same activations), the
output stays N-sharded; there is no collective inside the timed step.

Extra objects on the JSON line:
  roofline      the GEMM kernel against the int8 dense peak derived from the
                measured bf16 peak (2x, MEASURED_PEAKS.json)
  smoothquant   GB/s of b2sq_smoothquant at the prefill activation shape
                16384 x 8192 (reference byte formula, rocwmma_smoothquant.cpp:157-158)
  e2e           the same GEMM through the C ABI from pinned host buffers:
                H2D of A, B and scales + GEMM + D2H of C inside the timed region
  cpu_baseline  the CPU oracle (restated reference CPU path) on a row sample

``--impl reference`` times the reference's CPU path (the oracle restatement;
the HIP reference cannot run on this machine) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
M = N = K = 8192
FLUSH_BYTES = 512 << 20
SQ_M, SQ_K = 16384, 8192

# DRAM bytes (read + write) of one gemm_i8_pair_kernel launch at 8192^3, from
# the ncu capture summarised in profiles/gemm_i8_pair_8192_ncu.md.
GEMM_TRAFFIC_BYTES = 341_518_592  # 225,995,776 read + 115,522,816 written


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--profile", choices=["gemm", "smoothquant", "decode16", "decode64"], default=None,
                    help="run 3 launches of one kernel on its workload and exit (for ncu captures)")
    return ap.parse_args()


def run_profile(kind: str):
    """Three launches of one kernel at its workload size, nothing else (ncu target)."""
    import torch

    sys.path.insert(0, str(ROOT))
    from optimized_rocwmma_samples_b200 import api, synth

    dev = torch.device("cuda", 0)
    if kind == "smoothquant":
        x = torch.randn((SQ_M, SQ_K), device=dev).to(torch.float16)
        s = torch.ones((SQ_K,), device=dev)
        for _ in range(3):
            api.smoothquant(x, s)
    else:
        m = {"gemm": M, "decode16": 16, "decode64": 64}[kind]
        n = N if kind == "gemm" else 28672
        a = synth.torch_int8_uniform((m, K), dev, 1)
        w = synth.torch_int8_uniform((n, K), dev, 2)
        sa, sb = synth.torch_scales(m, dev, 3), synth.torch_scales(n, dev, 4)
        dt = torch.bfloat16 if kind == "gemm" else torch.float16
        for _ in range(3):
            api.gemm_quant(a, w.t(), sa, sb, out_dtype=dt)
    torch.cuda.synchronize()
    print(f"profile {kind}: 3 launches done")


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """Samples SM clock and throttle reasons every 20 ms on a thread."""

    REASONS = {
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, local_rank: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[local_rank]) if vis else local_rank
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
        except Exception:  # NVML unavailable: clocks reported as null
            self._h = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- CPU oracle
def cpu_gemm_sample(budget_s: float, seed: int = 0):
    """Times the oracle's int8 GEMM (+ dequant) on a row sample of the 8192^3
    workload; returns (TOPS, rows, seconds, threads)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)  # [N, K] K-major
    sb = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    rows = 4
    while True:
        a = rng.integers(-127, 128, size=(rows, K), dtype=np.int8)
        sa = rng.uniform(1e-3, 1e-2, rows).astype(np.float32)
        t0 = time.perf_counter()
        O.gemm_quant(a, w.T, sa, sb, out_dtype="bf16")
        dt = time.perf_counter() - t0
        if dt >= budget_s * 0.5 or rows >= M:
            return 2.0 * rows * N * K / dt / 1e12, rows, dt, O.num_threads()
        rows = min(M, max(rows * 2, int(rows * budget_s / max(dt, 1e-3))))


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    total_steps = args.steps + args.warmup
    per_step = max(0.5, min(3.0, 150.0 / max(total_steps, 1)))
    times, rows_used, thr = [], 0, 1
    for i in range(total_steps):
        tops, rows, dt, thr = cpu_gemm_sample(per_step, seed=i)
        if i >= args.warmup:
            times.append(tops)
            rows_used = rows
    value = statistics.median(times)
    sample = f"{rows_used} of {M} rows of the {M}x{N}x{K} int8 GEMM + bf16 dequant per step, oracle (gcc -O3 OpenMP)"
    line = {
        "impl": "reference", "metric": "int8 GEMM TOPS at 8192^3 (M=N=K=8192, bf16 out)", "value": value,
        "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8->int32",
        "data": "synthetic", "config": {"workload": "c2_square_int8_gemm_8192", "M": M, "N": N, "K": K,
                                         "parallelism": "cpu-reference"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": thr, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is HIP/rocWMMA (AMD only): its CPU path is restated in oracle/ and timed here",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.profile:
        return run_profile(args.profile)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from optimized_rocwmma_samples_b200 import api, synth

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    hbm_gbs, bf16_tflops, peak_src = measured_peaks()
    int8_peak = 2.0 * bf16_tflops

    # inputs: same activations on every rank, a distinct weight shard per rank
    a = synth.torch_int8_uniform((M, K), dev, 11)
    w = synth.torch_int8_uniform((N, K), dev, 100 + rank)  # [N_shard, K] K-major
    b = w.t()
    sa = synth.torch_scales(M, dev, 13)
    sb = synth.torch_scales(N, dev, 200 + rank)
    c = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    flush_buf = torch.ones(FLUSH_BYTES // 8, dtype=torch.int64, device=dev)

    def l2_flush():
        flush_buf.sum()
    ws = api.Workspace()
    stream = torch.cuda.current_stream(dev)

    def step():
        api.gemm_quant(a, b, sa, sb, out_dtype=torch.bfloat16, c=c, workspace=ws)

    for _ in range(max(args.warmup, 3)):
        l2_flush()
        step()
    torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        t_wall = time.perf_counter()
        for e0, e1 in evs:
            l2_flush()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
    barrier()
    if api.last_device_error() != 0:
        raise RuntimeError("a bounded device wait timed out during the benchmark")
    step_ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    ms = statistics.mean(step_ms)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ops = 2.0 * M * N * K
    value = world * ops / (ms_max * 1e-3) / 1e12
    achieved = ops / (ms * 1e-3) / 1e12

    # ---------------- smoothquant at the prefill activation shape (HBM bound)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    x = torch.randn((SQ_M, SQ_K), generator=g, device=dev).to(torch.float16)
    s = torch.empty((SQ_K,), device=dev).uniform_(0.5, 2.0, generator=g)
    y = torch.empty((SQ_M, SQ_K), dtype=torch.int8, device=dev)
    rs = torch.empty((SQ_M,), dtype=torch.float32, device=dev)
    for _ in range(5):
        api.smoothquant(x, s, y=y, row_scale=rs)
    sq_ms = []
    for _ in range(50):
        l2_flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        api.smoothquant(x, s, y=y, row_scale=rs)
        e1.record(stream)
        sq_ms.append((e0, e1))
    torch.cuda.synchronize()
    sq_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in sq_ms)
    sq_bytes = SQ_M * SQ_K * 2 + SQ_M * SQ_K + SQ_K * 4 + SQ_M * 4
    sq_gbs = sq_bytes / (sq_ms * 1e-3) / 1e9
    del x, y

    def timed(fn, n):
        """Mean device ms of fn over n steps (L2 flushed before each), max over ranks."""
        for _ in range(3):
            fn()
        evs = []
        barrier()
        for _ in range(n):
            l2_flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        t_ = torch.tensor([statistics.mean(a.elapsed_time(b) for a, b in evs)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        return float(t_.item())

    # ---------------- config 3: decode smoothquant + GEMM, HBM bound
    decode = {}
    w_dec = synth.torch_int8_uniform((28672, K), dev, 31)
    sb_dec = synth.torch_scales(28672, dev, 32)
    s_dec = torch.empty((K,), device=dev).uniform_(0.5, 2.0, generator=g)
    for md in (16, 64):
        x_dec = torch.randn((md, K), generator=g, device=dev).to(torch.float16)
        y_dec = torch.empty((md, K), dtype=torch.int8, device=dev)
        r_dec = torch.empty((md,), dtype=torch.float32, device=dev)
        o_dec = torch.empty((md, 28672), dtype=torch.float16, device=dev)

        def dec_step():  # one fused call: smoothquant, then the GEMM launched with PDL
            api.smoothquant_gemm(x_dec, s_dec, w_dec, sb_dec, out_dtype=torch.float16, xq=y_dec, row_scale=r_dec,
                                 c=o_dec, workspace=ws)

        ms_d = timed(dec_step, 50)
        bytes_d = (md * K * 2 + md * K + K * 4 + md * 4) + (md * K + 28672 * K + 4 * 28672 + 4 * md + 2 * md * 28672)
        decode[f"m{md}"] = {"ms": ms_d, "gbs": world * bytes_d / (ms_d * 1e-3) / 1e9,
                            "frac_of_measured_hbm": bytes_d / (ms_d * 1e-3) / 1e9 / hbm_gbs,
                            "shape": [md, K, 28672], "gpu_launches_per_step": 2}
    del w_dec

    # ---------------- config 4: N-sharded prefill (smoothquant + GEMM), 16384 x 8192 x 28672
    from optimized_rocwmma_samples_b200.sharded import ShardedPrefill, cuda_ops, shard_range

    PM, PN = 16384, 28672
    n0, n1 = shard_range(PN, world, rank)
    w_pf = synth.torch_int8_uniform((n1 - n0, K), dev, 40 + rank)
    sb_pf = synth.torch_scales(n1 - n0, dev, 50 + rank)
    layer = ShardedPrefill(w_pf, sb_pf, PN, cuda_ops(torch.bfloat16))
    x_pf = torch.randn((PM, K), generator=g, device=dev).to(torch.float16)
    s_pf = torch.empty((K,), device=dev).uniform_(0.5, 2.0, generator=g)
    ops_pf = 2.0 * PM * PN * K
    ms_pf = timed(lambda: layer.forward(x_pf, s_pf, PM, K, "replicated", False), 10)
    xq_pf, rs_pf = api.smoothquant(x_pf, s_pf)
    ms_gm = timed(lambda: layer.ops.gemm(xq_pf, layer.w, rs_pf, layer.sb), 10)
    prefill = {"shape": [PM, K, PN], "shard_cols": n1 - n0,
               "sharded_compute": {"ms": ms_pf, "tops": ops_pf / (ms_pf * 1e-3) / 1e12,
                                   "note": "x replicated, each rank quantises and multiplies its N shard, "
                                           "output left N-sharded"},
               "sharded_gemm": {"ms": ms_gm, "tops": ops_pf / (ms_gm * 1e-3) / 1e12,
                                "note": "the GEMM alone on each rank's N shard (max over ranks); "
                                        "scaling = the 1-GPU ms / this"}}
    del xq_pf, rs_pf
    if world > 1:
        ms_e = timed(lambda: layer.forward(x_pf if rank == 0 else None, s_pf, PM, K, "rank0", True), 5)
        prefill["with_collectives"] = {"ms": ms_e, "tops": ops_pf / (ms_e * 1e-3) / 1e12,
                                       "note": "rank 0 quantises, NCCL broadcast of Xq and row scales, "
                                               "sharded GEMM, NCCL all-gather of the bf16 output into [M, N]"}
        # GEMM -> all-gather of the output: NCCL after the GEMM vs fused into the GEMM's epilogue
        ms_g = timed(lambda: layer.forward(x_pf, s_pf, PM, K, "replicated", True), 5)
        ms_f = timed(lambda: layer.forward(x_pf, s_pf, PM, K, "replicated", "fused"), 5)
        from optimized_rocwmma_samples_b200.sharded import multicast_supported
        mc = multicast_supported(dev)
        ms_fm = None
        if mc:
            layer_mc = ShardedPrefill(w_pf, sb_pf, PN, cuda_ops(torch.bfloat16, gather="multicast"))
            ms_fm = timed(lambda: layer_mc.forward(x_pf, s_pf, PM, K, "replicated", "fused"), 5)
            layer_mc.ops.close()
            del layer_mc
        out_bytes = PM * PN * 2
        prefill["gather_nccl"] = {"ms": ms_g, "tops": ops_pf / (ms_g * 1e-3) / 1e12,
                                  "note": "x replicated, sharded GEMM, then NCCL all-gather into [M, N]"}
        prefill["gather_fused"] = {"ms": ms_f, "tops": ops_pf / (ms_f * 1e-3) / 1e12,
                                   "nvlink_bytes_out_per_gpu": out_bytes // world * (world - 1),
                                   "nvlink_bytes_in_per_gpu": out_bytes // world * (world - 1),
                                   "note": "x replicated, b2sq_gemm_i8_allgather: one GEMM whose epilogue stores "
                                           "every output tile into each rank's [M, N] buffer over NVLink (CUDA IPC "
                                           "mappings); one-element all-reduce barriers before and after"}
        if ms_fm is not None:
            prefill["gather_fused_multicast"] = {
                "ms": ms_fm, "tops": ops_pf / (ms_fm * 1e-3) / 1e12,
                "nvlink_bytes_out_per_gpu": out_bytes // world,
                "note": "b2sq_gemm_i8_allgather_mc: each output piece stored once with multimem.st through "
                        "the NVSwitch multicast mapping (torch symmetric memory); bound like the other by "
                        "the bytes every GPU receives"}
    layer.ops.close()
    del layer, w_pf, x_pf

    # ---------------- config 5: MoE, router -> sorting -> MoE smoothquant -> grouped GEMM (replicas)
    T5, H5, E5, K5, N5 = synth.MOE_TOKENS, synth.MOE_HIDDEN, synth.MOE_EXPERTS, synth.MOE_TOPK, synth.MOE_INTER
    logits5 = torch.randn((T5, E5), generator=g, device=dev).to(torch.float16)
    x5 = torch.randn((T5, H5), generator=g, device=dev).to(torch.float16)
    s5 = torch.empty((E5, H5), device=dev).uniform_(0.5, 2.0, generator=g)
    w5 = synth.torch_int8_uniform((E5, N5, H5), dev, 55)
    sb5 = synth.torch_scales(E5 * N5, dev, 56)
    unit5 = 128  # expert segments padded to whole 128-row tiles
    tw5, ti5 = api.topk_softmax(logits5, K5)
    cnt5, st5, sid5, perm5 = api.moe_sorting(ti5, E5, unit5)
    rows5 = T5 * K5 + E5 * unit5
    qy5 = torch.zeros((rows5, H5), dtype=torch.int8, device=dev)
    rs5 = torch.zeros((rows5,), dtype=torch.float32, device=dev)
    out5 = torch.empty((rows5, N5), dtype=torch.bfloat16, device=dev)

    def moe_step():
        api.topk_softmax(logits5, K5, tw5, ti5)
        cnt, st, _, perm = api.moe_sorting(ti5, E5, unit5)
        api.moe_smoothquant(x5, s5, ti5, qy=qy5, row_scale=rs5, row_perm=perm, out_rows=rows5)
        api.gemm_grouped(qy5, w5, st, cnt, rs5, sb5, out_dtype=torch.bfloat16, c=out5)

    ms_moe = timed(moe_step, 10)
    ms_grp = timed(lambda: api.gemm_grouped(qy5, w5, st5, cnt5, rs5, sb5, out_dtype=torch.bfloat16, c=out5), 10)
    ops5 = 2.0 * T5 * K5 * N5 * H5
    moe = {"shape": {"tokens": T5, "hidden": H5, "experts": E5, "topk": K5, "inter": N5},
           "pipeline_ms": ms_moe, "grouped_gemm_ms": ms_grp,
           "grouped_gemm_tops": ops5 / (ms_grp * 1e-3) / 1e12, "pipeline_tops": ops5 / (ms_moe * 1e-3) / 1e12,
           "gpu_launches_per_step": 4,
           "note": "router (b2sq_topk_softmax) -> b2sq_moe_sorting -> MoE smoothquant into expert order -> "
                   "b2sq_gemm_i8_grouped, all on the device; replicas at N > 1"}
    del w5, qy5, out5

    # ---------------- e2e through the C ABI from pinned host buffers
    h_a = a.cpu().pin_memory()
    h_w = w.cpu().pin_memory()
    h_sa = sa.cpu().pin_memory()
    h_sb = sb.cpu().pin_memory()
    h_c = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 10))
    e2e_bufs = [None]

    def e2e_step():
        # the public host-buffer call: weights once, activations in row chunks whose copies in,
        # GEMMs and copies out overlap (all inputs and the result cross PCIe every step)
        e2e_bufs[0] = api.gemm_quant_host(h_a, h_w, h_sa, h_sb, h_c, out_dtype=torch.bfloat16,
                                          buffers=e2e_bufs[0], workspace=ws)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = world * ops / (float(t.item()) * 1e-3) / 1e12
    h2d = a.numel() + w.numel() + 4 * (sa.numel() + sb.numel())
    d2h = c.numel() * 2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tops, rows, dt, thr = cpu_gemm_sample(10.0)
        cpu = {"value": tops, "unit": "TOPS", "cores": thr, "kind": "port",
               "sample": f"{rows} of {M} rows of the 8192^3 int8 GEMM + bf16 dequant ({dt:.1f} s), "
                         "oracle restating the reference CPU path (gcc -O3, OpenMP)"}

    if rank == 0:
        line = {
            "metric": "int8 GEMM TOPS at 8192^3 (M=N=K=8192, bf16 out)",
            "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8->int32", "data": "synthetic",
            "config": {"workload": "c2_square_int8_gemm_8192", "M": M, "N": N, "K": K,
                       "a_layout": "row-major", "b_layout": "column-major (K-major weights)",
                       "scales": "per-row x per-column fp32", "out": "bf16",
                       "parallelism": f"n-sharded x{world}" if world > 1 else "single-gpu",
                       "l2": "flushed (512 MB read) before every timed step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                         "frac": achieved / int8_peak, "traffic": GEMM_TRAFFIC_BYTES,
                         "peak_note": f"2 x {peak_src} bf16 dense {bf16_tflops} TFLOP/s (int8 dense rate = 2x bf16); "
                                      f"nominal int8 4500 TOPS -> frac {achieved / 4500.0:.3f}"},
            "smoothquant": {"shape": [SQ_M, SQ_K], "ms": sq_ms, "gbs": sq_gbs,
                            "frac_of_measured_hbm": sq_gbs / hbm_gbs, "hbm_peak_gbs": hbm_gbs},
            "decode": decode,
            "prefill_c4": prefill,
            "moe_c5": moe,
            "e2e": {"value": e2e_value, "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "wall_s_timed": t_wall,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
