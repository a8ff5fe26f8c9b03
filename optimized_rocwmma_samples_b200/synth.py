"""Seeded synthetic inputs with the shapes and distributions of the workload
configurations (the reference benchmarks constant inputs only; these stand in
for real activations/weights, which are not available offline).

numpy generators (CPU, for parity tests) and torch generators (on device, for
the benchmark) draw from the same distributions:
  activations x  ~ N(0, 1) in fp32, a few outlier channels scaled, rounded to fp16 once
  smooth scale   ~ U[0.5, 2]      fp32, per channel (per expert for MoE)
  weights W      ~ U{-127..127}   int8
  per-row/col dequant scales ~ U[1e-3, 1e-2] fp32
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    M: int
    K: int
    N: int
    outlier_cols: int
    outlier_scale: float
    out_dtype: str  # "f16" | "bf16"
    seed: int


# The five workload configurations (activations [M, K], weights [K, N]).
C1 = Config("c1_cpu_reference", 256, 1024, 512, 8, 20.0, "f16", 0)
C2 = Config("c2_square_8192", 8192, 8192, 8192, 0, 1.0, "bf16", 1)
C3_16 = Config("c3_decode_m16", 16, 8192, 28672, 8, 30.0, "f16", 2)
C3_64 = Config("c3_decode_m64", 64, 8192, 28672, 8, 30.0, "f16", 2)
C4 = Config("c4_prefill_16384", 16384, 8192, 28672, 8, 20.0, "bf16", 3)
# MoE: 4096 tokens x hidden 4096, 8 experts, top-2, expert W [4096, 14336].
MOE_TOKENS, MOE_HIDDEN, MOE_EXPERTS, MOE_TOPK, MOE_INTER = 4096, 4096, 8, 2, 14336
MOE_SEED = 4


def activations_np(rng: np.random.Generator, M: int, K: int, outlier_cols: int, outlier_scale: float) -> np.ndarray:
    x = rng.standard_normal((M, K), dtype=np.float32)
    if outlier_cols:
        cols = rng.choice(K, size=min(outlier_cols, K), replace=False)
        x[:, cols] *= np.float32(outlier_scale)
    return x.astype(np.float16)


def smooth_np(rng, K: int, rows: int | None = None) -> np.ndarray:
    shape = (K,) if rows is None else (rows, K)
    return rng.uniform(0.5, 2.0, size=shape).astype(np.float32)


def weights_np(rng, rows: int, cols: int) -> np.ndarray:
    return rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)


def scales_np(rng, n: int) -> np.ndarray:
    return rng.uniform(1e-3, 1e-2, size=(n,)).astype(np.float32)


def topk_routing_np(rng, tokens: int, experts: int, topk: int) -> np.ndarray:
    """softmax(N(0,1) logits) -> top-k expert ids.  Continuous logits have no
    ties; the device router (b2sq_topk_softmax) is the exact counterpart."""
    logits = rng.standard_normal((tokens, experts), dtype=np.float32)
    z = np.exp(logits - logits.max(axis=1, keepdims=True))
    p = z / z.sum(axis=1, keepdims=True)
    # stable sort on -p keeps lower ids first among equal probabilities
    order = np.argsort(-p, axis=1, kind="stable")
    return order[:, :topk].astype(np.int32)


def config_inputs_np(cfg: Config, M: int | None = None):
    """(x fp16 [M,K], smooth fp32 [K], W int8 [N,K] K-major storage, sb fp32 [N])."""
    rng = np.random.default_rng(cfg.seed)
    M = cfg.M if M is None else M
    x = activations_np(rng, M, cfg.K, cfg.outlier_cols, cfg.outlier_scale)
    s = smooth_np(rng, cfg.K)
    w_nk = weights_np(rng, cfg.N, cfg.K)
    sb = scales_np(rng, cfg.N)
    return x, s, w_nk, sb


# ---------------------------------------------------------------- torch (device)
def torch_inputs(cfg: Config, device, M: int | None = None):
    """Device-resident inputs of a configuration, drawn on the GPU."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed)
    M = cfg.M if M is None else M
    x = torch.randn((M, cfg.K), generator=g, device=device, dtype=torch.float32)
    if cfg.outlier_cols:
        cols = torch.randperm(cfg.K, generator=g, device=device)[: cfg.outlier_cols]
        x[:, cols] *= cfg.outlier_scale
    x = x.to(torch.float16)
    s = torch.empty((cfg.K,), device=device).uniform_(0.5, 2.0, generator=g)
    w_nk = torch.randint(-127, 128, (cfg.N, cfg.K), generator=g, device=device, dtype=torch.int8)
    sb = torch.empty((cfg.N,), device=device).uniform_(1e-3, 1e-2, generator=g)
    return x, s, w_nk, sb


def torch_int8_uniform(shape, device, seed: int):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, device=device, dtype=torch.int8)


def torch_scales(n: int, device, seed: int):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.empty((n,), device=device).uniform_(1e-3, 1e-2, generator=g)
