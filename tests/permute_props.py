"""Size-independent properties of a permute result (moe_permute's contract,
tests/test_reference.py:534-558 of the reference): expert-sorted, stable,
the two maps inverse to each other, offsets from the counts, and each
permuted row a bitwise copy of its token's row.  Plain torch, so the same
check runs on the oracle's output on the CPU and on the kernels' output at
full size on the GPU.  Test infrastructure only."""
from __future__ import annotations

import torch


def check_permute_properties(hidden, idx, E, permuted, offsets, s2d, perm):
    T, k = idx.shape
    dev = perm.device
    flat = idx.reshape(-1).to(dev).long()
    key = torch.where((flat < 0) | (flat >= E), torch.full_like(flat, E), flat)
    perm_l, s2d_l = perm.long(), s2d.long()
    sk = key[perm_l]
    assert bool((sk[1:] >= sk[:-1]).all()), "not sorted by expert"
    same = sk[1:] == sk[:-1]
    assert bool((perm_l[1:][same] > perm_l[:-1][same]).all()), "not stable"
    assert torch.equal(s2d_l[perm_l], torch.arange(T * k, device=dev)), "maps not inverse"
    counts = torch.bincount(key, minlength=E + 1)[:E]
    zero = torch.zeros(1, dtype=torch.long, device=dev)
    assert torch.equal(offsets.long(), torch.cat([zero, counts.cumsum(0)])), "offsets"
    if hidden is not None:
        assert torch.equal(permuted, hidden.to(dev)[perm_l // k]), "rows"
