"""B200-native (sm_100a) MoE expert kernels.

A from-scratch implementation of the MoE-layer hot path of
kkontosis/LayerStoRmExpertKernels: grouped top-k gating, permute/unpermute,
fused SwiGLU, the bf16 expert gate/up/down contraction (tcgen05/TMEM/TMA) and
the weighted (expert-parallel) combine.  The kernels live in liblsek.so behind
the C ABI of include/lsek.h; `_C` is the torch binding that exposes the
reference's operator surface (csrc/bindings_python.cu:371-417 of the
reference) under the same names.  `import sm120_expert_kernels` gives the same
module under the reference's name.

There is no CPU fallback: importing fails when the native extension has not
been built.  Build it with `python layerstormexpertkernels_b200/build.py`
(run as a script: `python -m` would execute this file first).
"""
from __future__ import annotations

import os

import torch  # noqa: F401  (loads libtorch before the binding)

_PKG = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_PKG, "liblsek.so")

try:
    from . import _C
except ImportError as exc:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "layerstormexpertkernels_b200: the native extension is not built "
        f"({exc}); run `python layerstormexpertkernels_b200/build.py`") from exc

from ._C import (  # noqa: E402,F401
    adaptive_gating,
    device_error,
    fused_swiglu,
    grouped_gemm_bf16,
    grouped_gemm_swiglu_bf16,
    moe_combine_reduce_slots_bf16_to_bf16,
    moe_combine_reduce_slots_fp32_to_bf16,
    moe_layer_forward_out,
    moe_layer_workspace_size,
    moe_permute,
    moe_route,
    moe_unpermute,
    moe_unpermute_bf16_perslot,
    moe_unpermute_fp32,
    topk_gating,
    version,
)
from .layer import (STAGES, HostPipeline, MoELayer, StageEvents, bind_host_to_device,  # noqa: E402,F401
                    moe_layer_forward)

__all__ = [
    "adaptive_gating", "device_error", "fused_swiglu", "grouped_gemm_bf16",
    "grouped_gemm_swiglu_bf16", "moe_combine_reduce_slots_bf16_to_bf16",
    "moe_combine_reduce_slots_fp32_to_bf16", "moe_layer_forward", "moe_layer_forward_out",
    "moe_layer_workspace_size", "moe_permute", "moe_route", "moe_unpermute", "moe_unpermute_bf16_perslot",
    "moe_unpermute_fp32", "topk_gating", "version", "MoELayer", "HostPipeline", "StageEvents", "bind_host_to_device",
    "STAGES",
    "LIBRARY_PATH",
]
