"""B200-native (sm_100a) smoothquant -> int8 GEMM hot path of optimized_rocwmma_samples.

The compute lives in ``libb2sq.so`` (CUDA kernels behind the C ABI of
``include/b2sq.h``); this package is its host-side mirror for Python callers.
"""
from .api import (  # noqa: F401
    B2sqError,
    COL_MAJOR,
    ROW_MAJOR,
    Workspace,
    debug_bounded_wait,
    gemm_quant,
    gemm_quant_host,
    gemm_quant_tensor_scale,
    kernel_moe_smoothquant,
    kernel_smoothquant,
    last_device_error,
    gemm_grouped,
    moe_smoothquant,
    moe_sorting,
    plan,
    smoothquant,
    smoothquant_gemm,
    topk_softmax,
    kernel_topk_softmax,
    workspace_size,
)

__version__ = "0.1.0"
