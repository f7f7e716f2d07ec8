"""Pins the CPU oracle to the reference: every oracle function against the
fixtures that tests/golden/make_golden.py produced by running the
reference's own torch implementation (tests/test_reference.py)."""
from __future__ import annotations

import os

import numpy as np
import pytest

import cases
from oracle import moe_oracle as O


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name + ".npz"))


@pytest.mark.parametrize("case", cases.GATING_CASES, ids=lambda c: c["name"])
def test_gating_matches_reference(golden_dir, case):
    d = load(golden_dir, "gating_" + case["name"])
    logits, bias = cases.gating_inputs(case)
    assert np.float64(logits.double().sum().item()) == d["logits_sum"], "input generator drifted"
    if "logits" in d:
        assert np.array_equal(d["logits"], logits.numpy())
    w, idx = O.topk_gating(logits.numpy(), None if bias is None else bias.numpy(), case["topk"],
                           case["n_group"], case["topk_group"], case["rsf"], case["renorm"],
                           case["scoring"])
    # Indices bit-exact, in selection order; weights within 1e-6 relative.
    assert np.array_equal(idx, d["indices"])
    rel = np.abs(w - d["weights"]) / np.maximum(np.abs(d["weights"]), np.float32(1e-30))
    assert rel.max() <= 1e-6, rel.max()


def test_gating_group_constraint_and_sum(golden_dir):
    c = cases.GATING_CASES[0]
    logits, bias = cases.gating_inputs(c)
    w, idx = O.topk_gating(logits.numpy(), bias.numpy(), 8, 8, 4, 2.5, True)
    groups = idx // 32
    assert all(len(set(r)) <= 4 for r in groups.tolist())
    assert np.allclose(w.sum(1), 2.5, atol=1e-5)


def test_sqrtsoftplus_known_values():
    x = np.array([0.0, -100.0, 100.0, 20.0, 20.5, -20.0], dtype=np.float32)
    s = O.sqrtsoftplus_scores(x)
    assert abs(s[0] - np.sqrt(np.log(2.0))) < 1e-6          # sqrt(ln 2)
    assert s[1] >= 0 and np.isfinite(s).all()
    assert s[2] == np.float32(10.0)                            # x > 20 -> sqrt(x)
    assert abs(s[5] - np.exp(-10.0)) / np.exp(-10.0) < 1e-5    # log1p keeps tiny values


def test_sigmoid_extremes_finite():
    s = O.sigmoid_scores(np.array([-100.0, 0.0, 100.0], np.float32))
    assert s[0] == 0.0 and s[1] == 0.5 and s[2] == 1.0


@pytest.mark.parametrize("name", ["known_answer", "rand64", "rand256_t05", "rand32_k4_t1"])
def test_adaptive_matches_reference(golden_dir, name):
    d = load(golden_dir, "adaptive_" + name)
    w, i, c = O.adaptive_gating(d["in_weights"], d["in_indices"], float(d["threshold"]))
    assert np.array_equal(c, d["counts"])
    assert np.array_equal(i, d["indices"])
    assert np.array_equal(w, d["weights"])


def test_adaptive_known_answer_counts(golden_dir):
    d = load(golden_dir, "adaptive_known_answer")
    _, i, c = O.adaptive_gating(d["in_weights"], d["in_indices"], 0.9)
    assert c.tolist() == [3, 1, 4, 3]
    assert i[0, 3] == -1 and (i[1, 1:] == -1).all()


@pytest.mark.parametrize("name", ["plain", "clamp10", "edges"])
def test_swiglu_matches_reference(golden_dir, name):
    d = load(golden_dir, "swiglu_" + name)
    out = O.swiglu(d["gate"], d["up"], float(d["limit"]))
    assert np.allclose(out, d["out"], rtol=1e-5, atol=1e-6)


def test_swiglu_clamp_semantics():
    # gate clamped from above only, up clamped both ways (ref_swiglu).
    g = np.array([-20.0, -10.0, 30.0], np.float32)
    u = np.array([1.0, 1.0, -100.0], np.float32)
    out = O.swiglu(g, u, 10.0)
    silu = lambda v: v / (1 + np.exp(-v))  # noqa: E731
    assert np.allclose(out, [silu(-20.0), silu(-10.0), silu(10.0) * -10.0])


@pytest.mark.parametrize("name", ["t128_k4_e32", "t96_k8_e64_sentinels", "t1_k8_e256",
                                  "t4096_k8_e256"])
def test_permute_matches_reference(golden_dir, name):
    d = load(golden_dir, "permute_" + name)
    _, offsets, s2d, perm = O.moe_permute(None, d["topk_indices"], int(d["num_experts"]))
    assert np.array_equal(perm, d["perm"])
    assert np.array_equal(s2d, d["s2d"])
    assert np.array_equal(offsets, d["offsets"])


def test_permute_round_trip_rows():
    rng = np.random.default_rng(0)
    hidden = rng.standard_normal((16, 8)).astype(np.float32)
    idx = rng.integers(0, 4, (16, 3)).astype(np.int32)
    permuted, _, s2d, _ = O.moe_permute(hidden, idx, 4)
    expanded = np.repeat(hidden, 3, axis=0)
    assert np.array_equal(permuted[s2d], expanded)


def test_combine_matches_reference(golden_dir):
    d = load(golden_dir, "combine_t24_k8_d256")
    T, k = d["weights"].shape
    x = O.bf16_from_bits(d["permuted"])
    f32 = O.moe_unpermute_perslot_f32(x, d["weights"], d["s2d"], T, k)
    assert np.array_equal(f32, d["perslot_f32"])
    b16 = O.moe_unpermute_perslot_bf16(x, d["weights"], d["s2d"], T, k)
    assert np.array_equal(O.bf16_bits(b16), d["perslot_bf16"])
    assert np.array_equal(O.bf16_bits(O.reduce_slots(f32)), d["reduce_f32"])
    assert np.array_equal(O.bf16_bits(O.reduce_slots(b16)), d["reduce_bf16"])


def test_unpermute_sum_is_fma_chain():
    rng = np.random.default_rng(1)
    T, k, H = 5, 4, 16
    x = O.bf16_round(rng.standard_normal((T * k, H)).astype(np.float32))
    w = rng.random((T, k)).astype(np.float32)
    s2d = rng.permutation(T * k).astype(np.int32)
    out = O.bf16_from_bits(O.moe_unpermute(O.bf16_bits(x), w, s2d, T, k))
    ref = np.zeros((T, H), np.float64)
    for t in range(T):
        for j in range(k):
            ref[t] += np.float64(w[t, j]) * x[s2d[t * k + j]]
    assert np.allclose(out, ref, rtol=1e-2, atol=1e-2)


def test_grouped_gemm_matches_reference(golden_dir):
    d = load(golden_dir, "grouped_gemm_e4")
    out = O.grouped_gemm(d["a"], d["b"], d["offsets"])
    assert np.allclose(out, d["out"], rtol=1e-5, atol=1e-4)


def test_expert_forward_top1_matches_reference(golden_dir):
    # ref_expert_forward with top-1 routing equals the layer composition with
    # topk = 1, weights = gating score, evaluated without bf16 stage rounding.
    d = load(golden_dir, "expert_forward_top1")
    x, ids, scores = d["x"], d["ids"], d["scores"]
    E = d["w_gate"].shape[0]
    _, offsets, s2d, perm = O.moe_permute(x, ids[:, None], E)
    w_gu = np.concatenate([d["w_gate"], d["w_up"]], axis=1)
    inter = d["w_gate"].shape[1]
    permuted = x[perm]
    y = np.zeros_like(permuted, dtype=np.float64)
    for e in range(E):
        s, t = offsets[e], offsets[e + 1]
        gu = permuted[s:t].astype(np.float64) @ w_gu[e].astype(np.float64).T
        h = O.swiglu(gu[:, :inter], gu[:, inter:])
        y[s:t] = h @ d["w_down"][e].astype(np.float64).T
    out = y[s2d] * scores[:, None]
    assert np.allclose(out, d["out"], rtol=1e-4, atol=1e-4)


# ---------------------------------------------------------------------------
# block-scaled weight formats (the next row of the hot-path scope)
# ---------------------------------------------------------------------------

def test_fp8_block_quant_matches_reference(golden_dir):
    from oracle import quant_oracle as Q
    d = load(golden_dir, "fp8_quant_m6_k300")
    q, scales = Q.dynamic_fp8_quant(d["x"])
    assert np.array_equal(scales.view(np.uint32), d["scales"].view(np.uint32))
    assert np.array_equal(q.view(np.uint32), d["q"].view(np.uint32))
    assert scales[2, 1] == 1.0  # the all-zero block
    deq = Q.fp8_dequant(d["q"], d["scales"])
    assert np.array_equal(deq.view(np.uint32), d["deq"].view(np.uint32))


def test_nvfp4_dequant_matches_reference(golden_dir):
    from oracle import quant_oracle as Q
    d = load(golden_dir, "nvfp4_dequant_m4_n64")
    out = Q.nvfp4_dequant(d["packed"], d["scales"])
    assert np.array_equal(out.view(np.uint32), d["out"].view(np.uint32))


def test_e4m3_codes_round_trip_and_known_values():
    from oracle import quant_oracle as Q
    codes = np.arange(256, dtype=np.uint8)
    vals = Q.e4m3_decode(codes)
    nan = np.isnan(vals)
    assert nan.sum() == 2 and nan[0x7F] and nan[0xFF]
    known = {0x00: 0.0, 0x01: 2.0 ** -9, 0x07: 7 * 2.0 ** -9, 0x08: 2.0 ** -6, 0x38: 1.0,
             0x3C: 1.5, 0x7E: 448.0, 0xB8: -1.0, 0xFE: -448.0}
    for c, v in known.items():
        assert vals[c] == np.float32(v), hex(c)
    finite = codes[~nan]
    assert np.array_equal(Q.e4m3_encode(vals[~nan]), finite)  # -0.0 keeps its sign code


def test_e4m3_rounding_is_nearest_even():
    from oracle import quant_oracle as Q
    pos = Q.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8)).astype(np.float64)
    mids = (pos[:-1] + pos[1:]) / 2.0
    got = Q.e4m3_encode(mids.astype(np.float32))
    lo_code = np.arange(0, 0x7E, dtype=np.uint8)
    want = np.where(lo_code % 2 == 0, lo_code, lo_code + 1).astype(np.uint8)
    assert np.array_equal(got, want)
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(20000) * np.exp2(rng.integers(-12, 9, 20000))).astype(np.float32)
    x = np.clip(x, -448, 448)
    r = Q.e4m3_round(x).astype(np.float64)
    allv = np.concatenate([-pos[::-1], pos])
    best = np.abs(allv[None, :] - x.astype(np.float64)[:, None]).min(axis=1)
    assert np.array_equal(np.abs(r - x), best)  # no representable value is nearer
    assert Q.e4m3_encode(np.float32(1000.0)) == 0x7E
    assert Q.e4m3_encode(np.float32(1000.0), saturate=False) == 0x7F
    assert Q.e4m3_encode(np.float32(464.0), saturate=False) == 0x7E  # the tie goes to 448
