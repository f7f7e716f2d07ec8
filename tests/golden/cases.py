"""Case definitions shared by tests/golden/make_golden.py and the tests that
read its fixtures: the parameters of every golden case and the seeded
generators of their inputs (torch CPU generator, fixed draw order)."""
from __future__ import annotations

import torch

# name, T, E, topk, n_group, topk_group, rsf, renorm, scoring, bias scale (None = no bias), seed
GATING_CASES = [
    dict(name="cfg0_grouped", T=128, E=256, topk=8, n_group=8, topk_group=4, rsf=2.5,
         renorm=True, scoring="sigmoid", bias_scale=0.01, seed=0),
    dict(name="t1024_grouped", T=1024, E=256, topk=8, n_group=8, topk_group=4, rsf=2.5,
         renorm=True, scoring="sigmoid", bias_scale=0.01, seed=1),
    dict(name="simple_bias", T=64, E=256, topk=8, n_group=1, topk_group=1, rsf=2.5,
         renorm=True, scoring="sigmoid", bias_scale=0.1, seed=2),
    dict(name="simple_norenorm", T=64, E=256, topk=8, n_group=1, topk_group=1, rsf=1.0,
         renorm=False, scoring="sigmoid", bias_scale=1.0, seed=3),
    dict(name="sqrtsoftplus_top6", T=64, E=256, topk=6, n_group=1, topk_group=1, rsf=2.5,
         renorm=True, scoring="sqrtsoftplus", bias_scale=0.1, seed=4),
    dict(name="v4_flat_top6_nobias", T=32, E=256, topk=6, n_group=1, topk_group=1, rsf=2.5,
         renorm=True, scoring="sqrtsoftplus", bias_scale=None, seed=5),
    dict(name="grouped_e64_top6", T=8, E=64, topk=6, n_group=8, topk_group=4, rsf=2.5,
         renorm=True, scoring="sigmoid", bias_scale=0.0, seed=6),
    dict(name="nobias_e64_top4", T=16, E=64, topk=4, n_group=1, topk_group=1, rsf=1.0,
         renorm=False, scoring="sigmoid", bias_scale=None, seed=7),
    dict(name="grouped_e128_g4", T=48, E=128, topk=6, n_group=4, topk_group=2, rsf=1.5,
         renorm=True, scoring="sqrtsoftplus", bias_scale=0.05, seed=8),
    dict(name="wide_logits", T=40, E=96, topk=5, n_group=1, topk_group=1, rsf=1.0,
         renorm=True, scoring="sigmoid", bias_scale=0.1, seed=9, logit_scale=8.0),
]


def gating_inputs(c):
    g = torch.Generator().manual_seed(c["seed"])
    logits = torch.randn(c["T"], c["E"], generator=g, dtype=torch.float32)
    logits = logits * c.get("logit_scale", 1.0)
    bias = None
    if c["bias_scale"] is not None:
        bias = torch.randn(c["E"], generator=g, dtype=torch.float32) * c["bias_scale"]
    return logits, bias


def adaptive_inputs(T, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.rand(T, k, generator=g, dtype=torch.float32)
    i = torch.randint(0, 256, (T, k), generator=g, dtype=torch.int32)
    return w, i


def permute_indices(T, k, E, sentinel_frac, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32)
    if sentinel_frac > 0:
        drop = torch.rand(T, k, generator=g) < sentinel_frac
        idx = torch.where(drop, torch.full_like(idx, -1), idx)
    return idx
