"""The EP steps restated on the CPU (oracle/ep_oracle.py wrapped in torch
tensors), with the same call signatures as layerstormexpertkernels_b200.ep
.DeviceSteps, so the EP host logic (splits, exchange order, combine) can run
over gloo without a GPU.  Test infrastructure only."""
from __future__ import annotations

import numpy as np
import torch

from oracle import ep_oracle as EO
from oracle import moe_oracle as MO


def _np(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy()


def _bf16(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def _i32(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))


class CpuSteps:
    @staticmethod
    def plan(topk_indices, num_experts, world_size):
        off, counts, pair_row, row_pair = EO.ep_plan(_np(topk_indices), num_experts, world_size)
        return _i32(off), _i32(counts), _i32(pair_row), _i32(row_pair)

    @staticmethod
    def dispatch_pack(hidden, topk_indices, topk_weights, pair_row, send_off, rows, num_experts,
                      world_size):
        r, ids, w = EO.ep_dispatch_pack(_np(hidden), _np(topk_indices), _np(topk_weights),
                                        _np(pair_row), _np(send_off), num_experts, world_size)
        assert r.shape[0] == rows
        return _bf16(r), _i32(ids), torch.from_numpy(w)

    @staticmethod
    def slot_scan(ids):
        return _i32(EO.ep_slot_scan(_np(ids)))

    @staticmethod
    def expert_permute(rows, local_ids, local_experts, valid_slots):
        p, off, s2d, perm = EO.ep_expert_permute(_np(rows), _np(local_ids), local_experts)
        assert p.shape[0] == valid_slots
        return _bf16(p), _i32(off), _i32(s2d), _i32(perm)

    @staticmethod
    def combine_pack(expert_out, s2d, ids, weights, slot_row, comb_rows):
        c = EO.ep_combine_pack(_np(expert_out), _np(s2d), _np(ids), _np(weights), _np(slot_row))
        assert c.shape[0] == comb_rows
        return _bf16(c)

    @staticmethod
    def combine_reduce(comb_rows, topk_indices, pair_row, slot_row, num_experts, world_size):
        return _bf16(EO.ep_combine_reduce(_np(comb_rows), _np(topk_indices), _np(pair_row),
                                          _np(slot_row), num_experts, world_size))

    @staticmethod
    def topk_gating(logits, bias, topk, n_group, topk_group, routed_scaling_factor, renormalize,
                    scoring_func="sigmoid"):
        w, idx = MO.topk_gating(_np(logits), None if bias is None else _np(bias), topk, n_group,
                                topk_group, routed_scaling_factor, renormalize, scoring_func)
        return torch.from_numpy(np.asarray(w, dtype=np.float32)), _i32(idx)

    @staticmethod
    def grouped_gemm_swiglu(a, w_gu, offsets, swiglu_limit=0.0):
        gu = MO.bf16_round(MO.grouped_gemm(_np(a), _np(w_gu), _np(offsets)).astype(np.float32))
        inter = gu.shape[1] // 2
        return _bf16(MO.swiglu(gu[:, :inter], gu[:, inter:], swiglu_limit).astype(np.float32))

    @staticmethod
    def grouped_gemm(a, b, offsets):
        return _bf16(MO.grouped_gemm(_np(a), _np(b), _np(offsets)).astype(np.float32))

    @staticmethod
    def moe_permute(hidden, topk_indices, num_experts):
        p, off, s2d, perm = MO.moe_permute(_np(hidden), _np(topk_indices), num_experts)
        return _bf16(p), _i32(off), _i32(s2d), _i32(perm)

    @staticmethod
    def unpermute_perslot(y, topk_weights, s2d, num_tokens, topk):
        return _bf16(MO.moe_unpermute_perslot_bf16(_np(y), _np(topk_weights), _np(s2d), num_tokens,
                                                   topk))

    @staticmethod
    def reduce_slots(perslot):
        return _bf16(MO.reduce_slots(_np(perslot)))


def canonical_layer(hidden, logits, bias, w_gu, w_down, topk=8, n_group=8, topk_group=4,
                    scale=2.5, renormalize=True):
    """One-rank reference of the EP layer: gating, permute, per-expert FFN
    with bf16 stage boundaries, then the canonical per-slot combine
    (moe_unpermute_bf16_perslot + moe_combine_reduce_slots_bf16_to_bf16).
    numpy in, fp32 values of bf16 out."""
    w, idx = MO.topk_gating(logits, bias, topk, n_group, topk_group, scale, renormalize)
    E = logits.shape[1]
    permuted, off, s2d, _ = MO.moe_permute(hidden, idx, E)
    y = np.zeros((permuted.shape[0], hidden.shape[1]), dtype=np.float32)
    for e in range(E):
        s, t = int(off[e]), int(off[e + 1])
        if t > s:
            y[s:t] = MO.expert_ffn(permuted[s:t], w_gu[e], w_down[e])
    T = hidden.shape[0]
    return MO.reduce_slots(MO.moe_unpermute_perslot_bf16(y, w, s2d, T, topk))
