"""Whole routed-expert layer: gating -> permute -> gate/up GEMM + SwiGLU ->
down GEMM -> weighted unpermute, as one call into liblsek
(lsek_moe_layer_forward).

The reference documents this flow (USAGE.md:40-57) but leaves the
composition to its caller; ref_expert_forward (tests/test_reference.py:257-276)
is its oracle for top-1 routing.
"""
from __future__ import annotations

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
