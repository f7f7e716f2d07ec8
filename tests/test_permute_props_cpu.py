"""The permute property checker against the oracle (so the checker the GPU
tests use at full size is itself checked), and that it catches a broken
result."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from oracle import moe_oracle as O
from permute_props import check_permute_properties


@pytest.mark.parametrize("T,k,E,sent", [(1, 1, 1, 0.0), (37, 8, 64, 0.1), (300, 6, 256, 0.0)])
def test_oracle_permute_has_the_properties(T, k, E, sent):
    idx = cases.permute_indices(T, k, E, sent, seed=T + k)
    hidden = torch.randn(T, 16)
    p, off, s2d, perm = O.moe_permute(hidden.numpy(), idx.numpy(), E)
    check_permute_properties(hidden, idx, E, torch.as_tensor(p), torch.as_tensor(off),
                             torch.as_tensor(s2d), torch.as_tensor(perm))


def test_checker_catches_an_unstable_order():
    idx = torch.tensor([[1, 1], [1, 0]], dtype=torch.int32)
    _, off, s2d, perm = O.moe_permute(None, idx.numpy(), 2)
    perm = torch.as_tensor(perm).clone()
    s2d = torch.as_tensor(s2d).clone()
    # swap the two slots of expert 1 that come first: sorted still, not stable
    perm[1], perm[2] = perm[2].clone(), perm[1].clone()
    s2d[perm.long()] = torch.arange(4, dtype=s2d.dtype)
    with pytest.raises(AssertionError, match="stable"):
        check_permute_properties(None, idx, 2, None, torch.as_tensor(off), s2d, perm)
