"""Seeded synthetic inputs with the shapes and distributions of the
DeepSeek-V3 MoE-layer configurations (no dataset is involved).

Draw order for token inputs, from torch.Generator().manual_seed(seed) on the
CPU: logits randn(T, E) f32; bias randn(E) * 0.01 f32; hidden randn(T, H)
cast to bf16.  Expert weights are drawn per expert from a generator seeded
with 1000 + e on the target device: W_gate, W_up [I, H] and W_down [H, I],
each randn * 0.02 cast to bf16, so any subset of experts can be regenerated
without materialising all of them.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HIDDEN = 7168
INTER = 2048
EXPERTS = 256
TOPK = 8
N_GROUP = 8
TOPK_GROUP = 4
ROUTED_SCALING = 2.5


@dataclass
class TokenInputs:
    logits: torch.Tensor   # [T, E] f32
    bias: torch.Tensor     # [E] f32
    hidden: torch.Tensor   # [T, H] bf16


def token_inputs(num_tokens: int, num_experts: int = EXPERTS, hidden_dim: int = HIDDEN,
                 seed: int = 0, device: str | torch.device = "cpu") -> TokenInputs:
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(num_tokens, num_experts, generator=g, dtype=torch.float32)
    bias = torch.randn(num_experts, generator=g, dtype=torch.float32) * 0.01
    hidden = torch.randn(num_tokens, hidden_dim, generator=g, dtype=torch.float32).to(torch.bfloat16)
    return TokenInputs(logits.to(device), bias.to(device), hidden.to(device))


def expert_weights(num_experts: int = EXPERTS, hidden_dim: int = HIDDEN, inter_dim: int = INTER,
                   device: str | torch.device = "cuda", seed_base: int = 1000,
                   experts: list[int] | None = None):
    """Returns (w_gu [E', 2I, H], w_down [E', H, I]) bf16 for `experts`
    (default: all), each expert drawn from its own generator."""
    device = torch.device(device)
    ids = list(range(num_experts)) if experts is None else list(experts)
    w_gu = torch.empty(len(ids), 2 * inter_dim, hidden_dim, dtype=torch.bfloat16, device=device)
    w_down = torch.empty(len(ids), hidden_dim, inter_dim, dtype=torch.bfloat16, device=device)
    for j, e in enumerate(ids):
        g = torch.Generator(device=device).manual_seed(seed_base + e)
        w_gu[j, :inter_dim] = torch.randn(inter_dim, hidden_dim, generator=g, device=device) * 0.02
        w_gu[j, inter_dim:] = torch.randn(inter_dim, hidden_dim, generator=g, device=device) * 0.02
        w_down[j] = torch.randn(hidden_dim, inter_dim, generator=g, device=device) * 0.02
    return w_gu, w_down
