"""Whole routed-expert layer: gating -> permute -> gate/up GEMM + SwiGLU ->
down GEMM -> weighted unpermute, as one call into liblsek
(lsek_moe_layer_forward).

The reference documents this flow (USAGE.md:40-57) but leaves the
composition to its caller; ref_expert_forward (tests/test_reference.py:257-276)
is its oracle for top-1 routing.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from . import _C


def moe_layer_forward(hidden: torch.Tensor, logits: torch.Tensor, bias: Optional[torch.Tensor],
                      w_gu: torch.Tensor, w_down: torch.Tensor, topk: int, n_group: int,
                      topk_group: int, routed_scaling_factor: float, renormalize: bool,
                      scoring_func: str = "sigmoid", swiglu_limit: float = 0.0,
                      return_routing: bool = False):
    """One MoE layer forward.

    hidden [T, H] bf16, logits [T, E] f32, bias [E] f32 or None,
    w_gu [E, 2I, H] bf16 (gate rows then up rows), w_down [E, H, I] bf16.
    Returns out [T, H] bf16, and (topk_weights, topk_indices) when
    return_routing is set.
    """
    T, H = hidden.shape
    E = logits.shape[1]
    inter = w_down.shape[2]
    ws = torch.empty(_C.moe_layer_workspace_size(T, H, inter, E, topk), dtype=torch.uint8,
                     device=hidden.device)
    out = torch.empty_like(hidden)
    w = idx = None
    if return_routing:
        w = torch.empty(T, topk, dtype=torch.float32, device=hidden.device)
        idx = torch.empty(T, topk, dtype=torch.int32, device=hidden.device)
    _C.moe_layer_forward_out(out, hidden, logits, bias, w_gu, w_down, topk, n_group, topk_group,
                             routed_scaling_factor, renormalize, scoring_func, swiglu_limit, ws,
                             w, idx)
    if return_routing:
        return out, w, idx
    return out


STAGES = ("gating", "route", "row_copy", "gate_up_swiglu_gemm", "down_gemm", "unpermute")


class StageEvents:
    """len(STAGES) + 1 timing events that lsek_moe_layer_forward records
    between its stages; elapsed_ms() gives the per-stage milliseconds."""

    def __init__(self):
        self._destroy = _C.events_destroy  # still callable while the interpreter shuts down
        self.handles = _C.events_create(len(STAGES) + 1)

    def elapsed_ms(self) -> dict:
        return dict(zip(STAGES, _C.events_elapsed_ms(self.handles)))

    def __del__(self):
        if getattr(self, "handles", None):
            self._destroy(self.handles)
            self.handles = []


class MoELayer:
    """A routed-expert layer with resident weights and a reusable workspace.

    The workspace grows to the largest token count seen and is reused, so a
    steady-state forward allocates only its output (or nothing, with `out=`),
    which keeps the call capturable in a CUDA graph.
    """

    def __init__(self, w_gu: torch.Tensor, w_down: torch.Tensor,
                 bias: Optional[torch.Tensor] = None, *, topk: int = 8, n_group: int = 8,
                 topk_group: int = 4, routed_scaling_factor: float = 2.5,
                 renormalize: bool = True, scoring_func: str = "sigmoid",
                 swiglu_limit: float = 0.0, max_tokens: int = 0):
        if w_gu.dim() != 3 or w_down.dim() != 3:
            raise ValueError("w_gu must be [E, 2I, H] and w_down [E, H, I]")
        self.w_gu, self.w_down, self.bias = w_gu, w_down, bias
        self.num_experts = w_gu.shape[0]
        self.hidden_dim = w_gu.shape[2]
        self.inter_dim = w_down.shape[2]
        self.topk, self.n_group, self.topk_group = topk, n_group, topk_group
        self.routed_scaling_factor = routed_scaling_factor
        self.renormalize = renormalize
        self.scoring_func = scoring_func
        self.swiglu_limit = swiglu_limit
        self.workspace = torch.empty(0, dtype=torch.uint8, device=w_gu.device)
        if max_tokens:
            self._ensure_workspace(max_tokens)

    def workspace_bytes(self, num_tokens: int) -> int:
        return _C.moe_layer_workspace_size(num_tokens, self.hidden_dim, self.inter_dim,
                                           self.num_experts, self.topk)

    def _ensure_workspace(self, num_tokens: int) -> None:
        need = self.workspace_bytes(num_tokens)
        if self.workspace.numel() < need:
            self.workspace = torch.empty(need, dtype=torch.uint8, device=self.w_gu.device)

    def forward(self, hidden: torch.Tensor, logits: torch.Tensor,
                out: Optional[torch.Tensor] = None,
                topk_weights: Optional[torch.Tensor] = None,
                topk_indices: Optional[torch.Tensor] = None,
                stage_events: Optional["StageEvents"] = None) -> torch.Tensor:
        """stage_events: None or a StageEvents, recorded on the current
        stream around the six stages (gating, route, row copy, gate/up GEMM +
        SwiGLU, down GEMM, unpermute)."""
        self._ensure_workspace(hidden.shape[0])
        if out is None:
            out = torch.empty_like(hidden)
        handles = [] if stage_events is None else stage_events.handles
        _C.moe_layer_forward_out(out, hidden, logits, self.bias, self.w_gu, self.w_down,
                                 self.topk, self.n_group, self.topk_group,
                                 self.routed_scaling_factor, self.renormalize, self.scoring_func,
                                 self.swiglu_limit, self.workspace, topk_weights, topk_indices,
                                 handles)
        return out

    __call__ = forward


def bind_host_to_device(device=None) -> Optional[list]:
    """Restricts the calling process to the CPU cores nearest `device` (the
    GPU's CPU affinity from NVML), so page-locked host buffers allocated
    afterwards live in the GPU's NUMA node and host<->device copies do not
    cross the socket link.  Returns the cores, or None (nothing changed) when
    NVML cannot tell.  Call it before allocating pinned buffers."""
    try:
        import pynvml
        idx = torch.device(device).index if device is not None else None
        if idx is None:
            idx = torch.cuda.current_device()
        props = torch.cuda.get_device_properties(idx)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        allowed = os.sched_getaffinity(0)
        cores = [64 * w + b for w, m in enumerate(mask) for b in range(64)
                 if (m >> b) & 1 and 64 * w + b in allowed]
        if not cores:
            return None
        os.sched_setaffinity(0, cores)
        return cores
    except Exception:  # no NVML, no GPU, or an affinity the OS refuses
        return None


class HostPipeline:
    """Feeds a layer from pinned host memory with the copies overlapped.

    `forward(hidden, logits)` runs on the current stream and returns the
    layer output (a device tensor).  submit() copies one batch from host to
    device on its own stream into one of `depth` device buffer sets, runs
    the layer once the copy has landed, and copies the output back to
    `out_host` on a third stream once the layer is done: while batch i
    computes, batch i+1 is being copied in and batch i-1 out.  Host buffers
    must be pinned; `out_host` holds its result after synchronize(), and an
    input host buffer can be refilled once the stream of the next submit()
    has copied it (after synchronize(), at the latest).  Allocate the pinned
    buffers after bind_host_to_device(), so they sit next to the GPU.
    """

    def __init__(self, forward, hidden_shape, logits_shape, device,
                 hidden_dtype=torch.bfloat16, logits_dtype=torch.float32, depth: int = 2):
        self.forward = forward
        self.depth = depth
        self.hidden = [torch.empty(hidden_shape, dtype=hidden_dtype, device=device)
                       for _ in range(depth)]
        self.logits = [torch.empty(logits_shape, dtype=logits_dtype, device=device)
                       for _ in range(depth)]
        self.h2d = torch.cuda.Stream(device=device)
        self.d2h = torch.cuda.Stream(device=device)
        self.copied_in = [torch.cuda.Event() for _ in range(depth)]
        self.computed = [torch.cuda.Event() for _ in range(depth)]
        self.used = [False] * depth
        self.count = 0

    def submit(self, hidden_host: torch.Tensor, logits_host: torch.Tensor,
               out_host: torch.Tensor) -> None:
        s = self.count % self.depth
        self.count += 1
        main = torch.cuda.current_stream()
        if self.used[s]:  # the layer that last read this buffer set has finished
            self.h2d.wait_event(self.computed[s])
        with torch.cuda.stream(self.h2d):
            self.hidden[s].copy_(hidden_host, non_blocking=True)
            self.logits[s].copy_(logits_host, non_blocking=True)
            self.copied_in[s].record(self.h2d)
        main.wait_event(self.copied_in[s])
        y = self.forward(self.hidden[s], self.logits[s])
        self.computed[s].record(main)
        self.used[s] = True
        self.d2h.wait_event(self.computed[s])
        with torch.cuda.stream(self.d2h):
            out_host.copy_(y, non_blocking=True)
        y.record_stream(self.d2h)  # keep the output's memory until the copy has read it

    def synchronize(self) -> None:
        self.d2h.synchronize()
        torch.cuda.current_stream().synchronize()
