"""CPU oracle for the MoE-layer hot path.

TEST INFRASTRUCTURE ONLY.  This module restates the reference's algorithms
(kkontosis/LayerStoRmExpertKernels) in numpy (+ a small C helper for fused
multiply-add chains) so the CUDA path can be checked against it.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
it; the product never does, and there is no CPU fallback in the product.

It is pinned against the reference itself: tests/golden/make_golden.py runs
the reference's own torch functions (tests/test_reference.py) and commits
their outputs as fixtures, and tests/test_oracle_golden.py checks every
function here against them.

Conventions.  16-bit activations travel as numpy float32 arrays holding
exactly representable bf16 values (or raw uint16 bit patterns where noted).
Every fp32 operation below is an explicit float32 numpy operation, so the
rounding sequence is the one written.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# 16-bit formats
# ---------------------------------------------------------------------------


def bf16_round(x) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 values."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))
         & np.uint32(0xFFFF0000))
    r = np.where(np.isnan(x), np.uint32(0x7FC00000), r).astype(np.uint32)
    return r.view(F32)


def bf16_bits(x) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_from_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(F32)


# ---------------------------------------------------------------------------
# Gating
# ---------------------------------------------------------------------------


def sigmoid_scores(logits) -> np.ndarray:
    """1 / (1 + e^-x) rounded to fp32 at each step: e^-x is evaluated in
    double and rounded once, then fp32 add and fp32 divide.  This is the
    formula of torch.sigmoid used by ref_topk_gating
    (tests/test_reference.py:148) without its single-precision exp
    approximation."""
    x = np.asarray(logits, dtype=F32)
    with np.errstate(over="ignore"):
        e = np.exp(-x.astype(np.float64)).astype(F32)
    return (F32(1.0) / (F32(1.0) + e)).astype(F32)


def sqrtsoftplus_scores(logits) -> np.ndarray:
    """sqrt(softplus(x)) with torch's softplus threshold (x > 20 -> x,
    else log1p(exp(x))), each step rounded to fp32; ref_sqrtsoftplus
    (tests/test_reference.py:128-130)."""
    x = np.asarray(logits, dtype=F32)
    big = x > F32(20.0)
    xs = np.where(big, F32(0.0), x)
    e = np.exp(xs.astype(np.float64)).astype(F32)
    lp = np.log1p(e.astype(np.float64)).astype(F32)
    return np.sqrt(np.where(big, x, lp)).astype(F32)


def topk_gating(logits, bias, topk: int, n_group: int = 1, topk_group: int = 1,
                routed_scaling_factor: float = 1.0, renormalize: bool = False,
                scoring_func: str = "sigmoid"):
    """Restates ref_topk_gating (tests/test_reference.py:133-187).

    Selection is on biased scores, weights are unbiased scores.  Grouped
    routing keeps the `topk_group` groups with the largest sum of their top-2
    biased scores (sm120/gating/topk_gating.cu:277-320 of the reference kernel).  Order and
    ties follow the reference kernel's packed keys (sm120/gating/topk_gating.cu:63-139):
    descending score, ties to the lower id (groups: to the lower group).  The
    renormalisation sum runs in selection order in fp32 and the scale is
    fp32 rsf / sum, as in warp_topk_select (topk_gating.cu:111-138).
    Returns (weights [T, topk] f32, indices [T, topk] int32)."""
    x = np.asarray(logits, dtype=F32)
    T, E = x.shape
    if scoring_func == "sigmoid":
        scores = sigmoid_scores(x)
    elif scoring_func == "sqrtsoftplus":
        scores = sqrtsoftplus_scores(x)
    else:
        raise ValueError(f"unknown scoring_func {scoring_func!r}")
    sel = (scores + np.asarray(bias, dtype=F32)[None, :]).astype(F32) if bias is not None \
        else scores.copy()
    cand = np.ones((T, E), dtype=bool)
    if n_group > 1:
        epg = E // n_group
        grp = sel.reshape(T, n_group, epg)
        desc = -np.sort(-grp, axis=2)
        gscore = (desc[:, :, 0] + desc[:, :, 1]).astype(F32) if epg >= 2 else desc[:, :, 0]
        order = np.argsort(-gscore, axis=1, kind="stable")
        kept = np.zeros((T, n_group), dtype=bool)
        np.put_along_axis(kept, order[:, :topk_group], True, axis=1)
        cand = np.repeat(kept, epg, axis=1)
    key = np.where(cand, -sel, np.inf)
    idx = np.argsort(key, axis=1, kind="stable")[:, :topk].astype(np.int32)
    w = np.take_along_axis(scores, idx.astype(np.int64), axis=1).astype(F32)
    if renormalize:
        s = np.zeros(T, dtype=F32)
        for k in range(topk):
            s = (s + w[:, k]).astype(F32)
        pos = s > F32(0.0)
        scale = (F32(routed_scaling_factor) / np.where(pos, s, F32(1.0))).astype(F32)
        w = np.where(pos[:, None], (w * scale[:, None]).astype(F32), w).astype(F32)
    return w, idx


def adaptive_gating(in_weights, in_indices, threshold: float):
    """Restates ref_adaptive_gating (tests/test_reference.py:190-225): per
    token, sort by weight descending (stable, as the reference kernel's
    insertion sort, adaptive_gating.cu:274-285), total = fp32 sum of the
    sorted weights, keep the shortest prefix whose running sum (double, as
    the reference's Python loop) reaches threshold * total, at least one.
    Returns (weights, indices, counts); dropped slots are (0.0, -1)."""
    w = np.asarray(in_weights, dtype=F32)
    i = np.asarray(in_indices, dtype=np.int32)
    T, K = w.shape
    order = np.argsort(-w, axis=1, kind="stable")
    sw = np.take_along_axis(w, order, axis=1)
    si = np.take_along_axis(i, order, axis=1)
    total = np.zeros(T, dtype=F32)
    for k in range(K):
        total = (total + sw[:, k]).astype(F32)
    target = float(threshold) * total.astype(np.float64)
    cum = np.cumsum(sw.astype(np.float64), axis=1)
    reached = cum >= target[:, None]
    count = np.where(reached.any(axis=1), reached.argmax(axis=1) + 1, K)
    count = np.maximum(count, 1).astype(np.int32)
    keep = np.arange(K)[None, :] < count[:, None]
    return (np.where(keep, sw, F32(0.0)).astype(F32), np.where(keep, si, -1).astype(np.int32),
            count)


# ---------------------------------------------------------------------------
# Permute / unpermute
# ---------------------------------------------------------------------------


def moe_permute(hidden, topk_indices, num_experts: int):
    """Stable expert-major permutation of the T*topk slots.

    Restates the permute of tests/test_reference.py:534-558
    (torch.argsort(flat, stable=True)) with the reference kernel's sentinel
    rule (smxx/permute/moe_permute.cu:47-61: an index < 0 sorts as expert E)
    and offsets (moe_permute.cu:66-92: offsets[e] = #slots with expert < e,
    e in [0, E]).  Any index outside [0, E) is treated as the sentinel.
    Returns (permuted rows or None, offsets [E+1], s2d [T*topk], perm [T*topk])."""
    idx = np.asarray(topk_indices)
    topk = idx.shape[1]
    flat = idx.reshape(-1).astype(np.int64)
    key = np.where((flat >= 0) & (flat < num_experts), flat, num_experts)
    perm = np.argsort(key, kind="stable").astype(np.int32)
    s2d = np.empty_like(perm)
    s2d[perm] = np.arange(perm.size, dtype=np.int32)
    counts = np.bincount(key[key < num_experts], minlength=num_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    permuted = None
    if hidden is not None:
        permuted = np.asarray(hidden)[perm.astype(np.int64) // max(topk, 1)]
    return permuted, offsets, s2d, perm


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        from . import build_oracle
        _LIB = ctypes.CDLL(build_oracle.build())
        _LIB.oracle_unpermute_sum.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
            ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p]
        _LIB.oracle_unpermute_sum.restype = None
    return _LIB


def moe_unpermute(permuted_bits, topk_weights, s2d, num_tokens: int, topk: int,
                  fp16: bool = False) -> np.ndarray:
    """out[t] = round16(sum_k fma(w[t,k], x[s2d[t,k]], acc)) in slot order
    (finalize_moe_routing_bf16, moe_permute.cu:182-246).  permuted_bits is
    uint16 [rows, H]; returns uint16 [T, H]."""
    x = np.ascontiguousarray(permuted_bits, dtype=np.uint16)
    w = np.ascontiguousarray(topk_weights, dtype=F32).reshape(-1)
    d = np.ascontiguousarray(s2d, dtype=np.int32).reshape(-1)
    H = x.shape[1]
    out = np.empty((num_tokens, H), dtype=np.uint16)
    _lib().oracle_unpermute_sum(x.ctypes.data, w.ctypes.data, d.ctypes.data, num_tokens, topk, H,
                                1 if fp16 else 0, out.ctypes.data)
    return out


def moe_unpermute_perslot_f32(permuted, topk_weights, s2d, num_tokens: int, topk: int):
    """out[t,k,:] = w[t,k] * x[s2d[t,k]] in fp32, no cross-slot sum
    (moe_permute.cu:330-376; tests/test_kernels.py:113-120)."""
    x = np.asarray(permuted, dtype=F32)
    w = np.asarray(topk_weights, dtype=F32).reshape(num_tokens, topk)
    d = np.asarray(s2d).reshape(num_tokens, topk).astype(np.int64)
    return (w[:, :, None] * x[d]).astype(F32)


def moe_unpermute_perslot_bf16(permuted, topk_weights, s2d, num_tokens: int, topk: int):
    """out[t,k,:] = bf16(w[t,k] * x[s2d[t,k]]) (moe_permute.cu:389-434;
    tests/test_kernels.py:168-176); returned as fp32 values."""
    return bf16_round(moe_unpermute_perslot_f32(permuted, topk_weights, s2d, num_tokens, topk))


def reduce_slots(perslot) -> np.ndarray:
    """bf16(((0 + in[:,0]) + in[:,1]) + ...) in fp32, fixed slot order
    (moe_permute.cu:440-474; tests/test_kernels.py:125-128); fp32 values."""
    p = np.asarray(perslot, dtype=F32)
    acc = np.zeros((p.shape[0], p.shape[2]), dtype=F32)
    for k in range(p.shape[1]):
        acc = (acc + p[:, k, :]).astype(F32)
    return bf16_round(acc)


# ---------------------------------------------------------------------------
# Activation and contraction
# ---------------------------------------------------------------------------


def swiglu(gate, up, swiglu_limit: float = 0.0) -> np.ndarray:
    """silu(g) * u with the clamp of ref_swiglu (tests/test_reference.py:110-125):
    g = min(g, L), u = clamp(u, -L, L) when L > 0.  Evaluated in double."""
    g = np.asarray(gate, dtype=np.float64)
    u = np.asarray(up, dtype=np.float64)
    if swiglu_limit > 0.0:
        g = np.minimum(g, swiglu_limit)
        u = np.clip(u, -swiglu_limit, swiglu_limit)
    with np.errstate(over="ignore"):
        return g / (1.0 + np.exp(-g)) * u


def grouped_gemm(a, b, expert_offsets) -> np.ndarray:
    """Restates ref_grouped_gemm (tests/test_reference.py:228-254):
    out[rows of e] = a[rows of e] @ b[e].T, evaluated in double; rows outside
    every expert stay zero.  a [rows, K], b [E, N, K]."""
    a = np.asarray(a, dtype=np.float64)
    offs = np.asarray(expert_offsets, dtype=np.int64)
    E, N = len(offs) - 1, np.asarray(b).shape[1]
    out = np.zeros((a.shape[0], N), dtype=np.float64)
    for e in range(E):
        s, t = offs[e], offs[e + 1]
        if t > s:
            out[s:t] = a[s:t] @ np.asarray(b[e], dtype=np.float64).T
    return out


def moe_layer_forward(hidden, logits, bias, w_gu, w_down, topk: int, n_group: int,
                      topk_group: int, routed_scaling_factor: float, renormalize: bool,
                      scoring_func: str = "sigmoid", swiglu_limit: float = 0.0):
    """The routed-expert layer as the GPU pipeline composes it (USAGE.md:40-57
    of the reference; ref_expert_forward, tests/test_reference.py:257-276,
    generalised to top-k): gating -> permute -> g,u = bf16(x @ W^T) ->
    h = bf16(swiglu(g, u)) -> y = bf16(h @ Wd^T) -> fma unpermute.  bf16
    rounding happens at the same stage boundaries as on the GPU; the GEMMs
    are evaluated in double.  hidden holds bf16 values as fp32; w_gu[e]
    ([2I, H]) and w_down[e] ([H, I]) are indexed per expert (arrays, or any
    object whose [e] yields one expert's weights, so callers can stream them).
    Returns (out bf16 bits [T, H], weights, indices)."""
    w, idx = topk_gating(logits, bias, topk, n_group, topk_group, routed_scaling_factor,
                         renormalize, scoring_func)
    E = np.asarray(logits).shape[1]
    permuted, offsets, s2d, _ = moe_permute(hidden, idx, E)
    H = np.asarray(hidden).shape[1]
    y = np.zeros((permuted.shape[0], H), dtype=F32)
    for e in range(E):
        s, t = int(offsets[e]), int(offsets[e + 1])
        if t <= s:
            continue
        y[s:t] = expert_ffn(permuted[s:t], w_gu[e], w_down[e], swiglu_limit)
    out = moe_unpermute(bf16_bits(y), w, s2d, idx.shape[0], topk)
    return out, w, idx


def expert_ffn(x, w_gu_e, w_down_e, swiglu_limit: float = 0.0, gemm_dtype=np.float64):
    """One expert on its rows with the GPU's bf16 stage boundaries:
    bf16(swiglu(bf16(x Wg^T), bf16(x Wu^T))) Wd^T -> bf16.  GEMMs in
    `gemm_dtype`: double for checking, fp32 (ref_grouped_gemm's precision,
    tests/test_reference.py:250-252) for the timed CPU baseline.  Returns
    fp32 values."""
    wgu = np.asarray(w_gu_e, dtype=gemm_dtype)
    inter = wgu.shape[0] // 2
    gu = bf16_round((np.asarray(x, dtype=gemm_dtype) @ wgu.T).astype(F32))
    h = bf16_round(swiglu(gu[:, :inter], gu[:, inter:], swiglu_limit).astype(F32))
    return bf16_round((h.astype(gemm_dtype) @ np.asarray(w_down_e, gemm_dtype).T).astype(F32))
