"""The drop-in operator surface, checked on the CPU: the module imports under
the reference's name, exposes the reference's ops with the same argument
names and defaults (csrc/bindings_python.cu:371-417 of the reference), and
rejects CPU tensors the way the reference's TORCH_CHECKs do."""
from __future__ import annotations

import re

import pytest
import torch

import sm120_expert_kernels as EK

# name -> [(argument, default or None)], from bindings_python.cu:371-417.
REFERENCE_OPS = {
    "fused_swiglu": [("input", None), ("swiglu_limit", "0.0")],
    "moe_permute": [("hidden_states", None), ("topk_indices", None), ("num_experts", None)],
    "moe_unpermute": [("permuted_output", None), ("topk_weights", None),
                      ("src_to_dest_map", None), ("num_tokens", None), ("topk", None)],
    "moe_unpermute_fp32": [("permuted_output", None), ("topk_weights", None),
                           ("src_to_dest_map", None), ("num_tokens", None), ("topk", None)],
    "moe_combine_reduce_slots_fp32_to_bf16": [("input_perslot_fp32", None)],
    "moe_unpermute_bf16_perslot": [("permuted_output", None), ("topk_weights", None),
                                   ("src_to_dest_map", None), ("num_tokens", None),
                                   ("topk", None)],
    "moe_combine_reduce_slots_bf16_to_bf16": [("input_perslot_bf16", None)],
    "adaptive_gating": [("in_weights", None), ("in_indices", None), ("threshold", None)],
    "topk_gating": [("logits", None), ("bias", None), ("topk", None), ("n_group", None),
                    ("topk_group", None), ("routed_scaling_factor", None),
                    ("renormalize", None), ("scoring_func", "'sigmoid'")],
}


def parse_signature(fn):
    first = fn.__doc__.splitlines()[0]
    args = first[first.index("(") + 1: first.rindex(") ->")]
    out = []
    for part in re.split(r",\s*(?=\w+:)", args):
        name, rest = part.split(":", 1)
        default = rest.split(" = ", 1)[1].strip() if " = " in rest else None
        out.append((name.strip(), default))
    return out


@pytest.mark.parametrize("name,expected", REFERENCE_OPS.items())
def test_reference_op_signatures(name, expected):
    assert parse_signature(getattr(EK, name)) == expected


def test_returns_documented_tuple_arity():
    assert "list[torch.Tensor]" in EK.moe_permute.__doc__.splitlines()[0]
    assert "list[torch.Tensor]" in EK.topk_gating.__doc__.splitlines()[0]


def test_native_library_is_the_product():
    import layerstormexpertkernels_b200 as P
    assert P.version().startswith("lsek ")
    assert P._C.__file__.endswith(".so")


@pytest.mark.parametrize("call", [
    lambda: EK.fused_swiglu(torch.zeros(4, 8, dtype=torch.bfloat16)),
    lambda: EK.moe_permute(torch.zeros(4, 8, dtype=torch.bfloat16),
                           torch.zeros(4, 2, dtype=torch.int32), 4),
    lambda: EK.topk_gating(torch.zeros(4, 8), None, 2, 1, 1, 1.0, False),
    lambda: EK.adaptive_gating(torch.zeros(4, 8), torch.zeros(4, 8, dtype=torch.int32), 0.5),
    lambda: EK.moe_combine_reduce_slots_fp32_to_bf16(torch.zeros(2, 2, 8)),
])
def test_cpu_tensors_rejected(call):
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        call()
