"""GPU parity of top-k gating and adaptive gating against the oracle (and, via
the oracle's golden pin, against the reference's ref_topk_gating /
ref_adaptive_gating).  Bar: indices bit-exact in selection order, weights
within 1e-6 relative; adaptive gating exact."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from gpu_util import dev
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def ek():
    import sm120_expert_kernels as EK
    return EK


def run_gating(logits, bias, c):
    w, idx = ek().topk_gating(dev(logits), None if bias is None else dev(bias), c["topk"],
                              c["n_group"], c["topk_group"], c["rsf"], c["renorm"], c["scoring"])
    torch.cuda.synchronize()
    return w.cpu().numpy(), idx.cpu().numpy()


def check_gating(w, idx, ow, oidx):
    assert np.array_equal(idx, oidx), f"{(idx != oidx).sum()} index mismatches"
    rel = np.abs(w - ow) / np.maximum(np.abs(ow), np.float32(1e-30))
    assert rel.max() <= 1e-6, rel.max()


@pytest.mark.parametrize("case", cases.GATING_CASES, ids=lambda c: c["name"])
def test_gating_golden_cases(case):
    logits, bias = cases.gating_inputs(case)
    lg = logits.numpy()
    b = None if bias is None else bias.numpy()
    w, idx = run_gating(lg, b, case)
    ow, oidx = O.topk_gating(lg, b, case["topk"], case["n_group"], case["topk_group"],
                             case["rsf"], case["renorm"], case["scoring"])
    check_gating(w, idx, ow, oidx)


@pytest.mark.parametrize("T", [1, 2, 3, 31, 33, 4096, 16384])
def test_gating_deepseek_shape(T):
    from layerstormexpertkernels_b200.synthetic import token_inputs
    x = token_inputs(T, hidden_dim=8, seed=100 + T)
    c = dict(topk=8, n_group=8, topk_group=4, rsf=2.5, renorm=True, scoring="sigmoid")
    w, idx = run_gating(x.logits.numpy(), x.bias.numpy(), c)
    ow, oidx = O.topk_gating(x.logits.numpy(), x.bias.numpy(), 8, 8, 4, 2.5, True)
    check_gating(w, idx, ow, oidx)
    assert np.allclose(w.sum(1), 2.5, atol=1e-5)
    assert all(len(set(r)) <= 4 for r in (idx // 32).tolist())


@pytest.mark.parametrize("E,n_group,topk_group,topk,scoring", [
    (8, 1, 1, 2, "sigmoid"), (32, 4, 2, 3, "sigmoid"), (48, 3, 2, 7, "sqrtsoftplus"),
    (100, 1, 1, 9, "sigmoid"), (160, 32, 5, 5, "sigmoid"), (384, 8, 3, 12, "sqrtsoftplus"),
    (512, 16, 8, 32, "sigmoid"), (1024, 32, 4, 16, "sigmoid"), (1000, 1, 1, 32, "sigmoid"),
])
def test_gating_shapes(E, n_group, topk_group, topk, scoring):
    g = torch.Generator().manual_seed(E * 7 + topk)
    logits = torch.randn(77, E, generator=g).numpy()
    bias = (torch.randn(E, generator=g) * 0.05).numpy()
    c = dict(topk=topk, n_group=n_group, topk_group=topk_group, rsf=1.7, renorm=True,
             scoring=scoring)
    w, idx = run_gating(logits, bias, c)
    ow, oidx = O.topk_gating(logits, bias, topk, n_group, topk_group, 1.7, True, scoring)
    check_gating(w, idx, ow, oidx)


def test_gating_ties_go_to_lower_id():
    # All-equal rows: the reference kernel's packed keys pick the lowest ids.
    logits = np.zeros((4, 64), np.float32)
    logits[1] = 3.0
    logits[2, 10:20] = 5.0
    c = dict(topk=6, n_group=8, topk_group=2, rsf=1.0, renorm=False, scoring="sigmoid")
    w, idx = run_gating(logits, None, c)
    ow, oidx = O.topk_gating(logits, None, 6, 8, 2, 1.0, False)
    check_gating(w, idx, ow, oidx)
    assert idx[0].tolist() == [0, 1, 2, 3, 4, 5]


def test_gating_ties_at_deepseek_shape():
    # E=256, 8 groups / 4 kept, top-8 (the register path, eight experts per
    # lane): equal scores pick the lowest groups, then the lowest ids.
    logits = np.zeros((3, 256), np.float32)
    logits[1, 200:] = 1.0          # one group's tail ahead, the rest tied
    logits[2, ::3] = -1.0
    c = dict(topk=8, n_group=8, topk_group=4, rsf=2.5, renorm=True, scoring="sigmoid")
    w, idx = run_gating(logits, None, c)
    ow, oidx = O.topk_gating(logits, None, 8, 8, 4, 2.5, True)
    check_gating(w, idx, ow, oidx)
    assert idx[0].tolist() == list(range(8))


def test_gating_sqrtsoftplus_extremes():
    # tests/test_topk_gating.py:274-297: large / small logits stay finite.
    logits = np.zeros((8, 64), np.float32)
    logits[0], logits[1] = 100.0, -100.0
    logits[3] = np.linspace(-50, 50, 64, dtype=np.float32)
    c = dict(topk=4, n_group=1, topk_group=1, rsf=1.0, renorm=False, scoring="sqrtsoftplus")
    w, idx = run_gating(logits, None, c)
    assert np.isfinite(w).all() and (w >= 0).all()
    ow, oidx = O.topk_gating(logits, None, 4, 1, 1, 1.0, False, "sqrtsoftplus")
    check_gating(w, idx, ow, oidx)


def test_gating_default_scoring_is_sigmoid():
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(64, 256, generator=g).cuda()
    bias = (torch.randn(256, generator=g) * 0.1).cuda()
    a = ek().topk_gating(logits, bias, 8, 1, 1, 2.5, True, scoring_func="sigmoid")
    b = ek().topk_gating(logits, bias, 8, 1, 1, 2.5, True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_gating_errors():
    logits = torch.randn(4, 64).cuda()
    with pytest.raises(RuntimeError, match="scoring_func"):
        ek().topk_gating(logits, None, 2, 1, 1, 1.0, False, scoring_func="softmax")
    with pytest.raises(ValueError, match="divisible"):
        ek().topk_gating(logits, None, 2, 7, 1, 1.0, False)
    with pytest.raises(ValueError, match="kept groups"):
        ek().topk_gating(logits, None, 40, 8, 4, 1.0, False)


def test_gating_zero_tokens():
    w, idx = ek().topk_gating(torch.empty(0, 256).cuda(), None, 8, 8, 4, 2.5, True)
    assert w.shape == (0, 8) and idx.shape == (0, 8)


@pytest.mark.parametrize("name", ["known_answer", "rand64", "rand256_t05", "rand32_k4_t1"])
def test_adaptive_golden(golden_dir, name):
    d = np.load(os.path.join(golden_dir, f"adaptive_{name}.npz"))
    w, i, c = ek().adaptive_gating(dev(d["in_weights"]), dev(d["in_indices"]), float(d["threshold"]))
    assert np.array_equal(c.cpu().numpy(), d["counts"])
    assert np.array_equal(i.cpu().numpy(), d["indices"])
    assert np.array_equal(w.cpu().numpy(), d["weights"])


@pytest.mark.parametrize("T,k,thr", [(1, 1, 0.5), (1000, 8, 0.9), (333, 16, 0.7), (64, 32, 0.0),
                                     (5, 3, 1.0)])
def test_adaptive_vs_oracle(T, k, thr):
    g = torch.Generator().manual_seed(T + k)
    w = torch.rand(T, k, generator=g)
    w[::7, 1:] = w[::7, :1]  # ties: stable order must be kept
    i = torch.randint(0, 256, (T, k), generator=g, dtype=torch.int32)
    gw, gi, gc = ek().adaptive_gating(w.cuda(), i.cuda(), thr)
    ow, oi, oc = O.adaptive_gating(w.numpy(), i.numpy(), thr)
    assert np.array_equal(gc.cpu().numpy(), oc)
    assert np.array_equal(gi.cpu().numpy(), oi)
    assert np.array_equal(gw.cpu().numpy(), ow)
