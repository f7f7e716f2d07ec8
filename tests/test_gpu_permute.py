"""GPU parity of permute, the unpermute family, the slot reduces and SwiGLU
against the oracle; all integer/byte results bit-exact, plus the reference's
own GPU test cases (tests/test_kernels.py, tests/test_fused_swiglu.py)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cases
from gpu_util import bits, dev
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def ek():
    import sm120_expert_kernels as EK
    return EK


def rand_bf16(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


# ---- permute -------------------------------------------------------------------

@pytest.mark.parametrize("name", ["t128_k4_e32", "t96_k8_e64_sentinels", "t1_k8_e256",
                                  "t4096_k8_e256"])
def test_permute_golden(golden_dir, name):
    d = np.load(os.path.join(golden_dir, f"permute_{name}.npz"))
    idx = d["topk_indices"]
    T = idx.shape[0]
    hidden = rand_bf16((T, 64), seed=T)
    p, off, s2d, perm = ek().moe_permute(hidden.cuda(), dev(idx), int(d["num_experts"]))
    assert np.array_equal(perm.cpu().numpy(), d["perm"])
    assert np.array_equal(s2d.cpu().numpy(), d["s2d"])
    assert np.array_equal(off.cpu().numpy(), d["offsets"])
    assert torch.equal(p.cpu(), hidden[torch.as_tensor(d["perm"]).long() // idx.shape[1]])


@pytest.mark.parametrize("T,k,E,H,sent", [
    (1, 1, 1, 8, 0.0), (2, 8, 256, 7168, 0.0), (31, 3, 5, 40, 0.2), (33, 8, 256, 100, 0.0),
    (128, 8, 256, 7168, 0.0), (4096, 8, 256, 256, 0.0), (4097, 8, 256, 64, 0.05),
    (8192, 8, 256, 128, 0.0), (20000, 6, 1023, 16, 0.01), (3, 32, 64, 24, 0.0),
])
def test_permute_vs_oracle(T, k, E, H, sent):
    idx = cases.permute_indices(T, k, E, sent, seed=T * 3 + k)
    hidden = rand_bf16((T, H), seed=T + H)
    p, off, s2d, perm = ek().moe_permute(hidden.cuda(), idx.cuda(), E)
    op, ooff, os2d, operm = O.moe_permute(bits(hidden), idx.numpy(), E)
    assert np.array_equal(perm.cpu().numpy(), operm)
    assert np.array_equal(s2d.cpu().numpy(), os2d)
    assert np.array_equal(off.cpu().numpy(), ooff)
    assert np.array_equal(bits(p), op)


def test_permute_out_of_range_indices_sort_last():
    idx = torch.tensor([[3, -1], [7, 0], [-5, 3]], dtype=torch.int32)  # 7 >= E
    hidden = rand_bf16((3, 16), seed=1)
    p, off, s2d, perm = ek().moe_permute(hidden.cuda(), idx.cuda(), 4)
    _, ooff, os2d, operm = O.moe_permute(None, idx.numpy(), 4)
    assert np.array_equal(off.cpu().numpy(), ooff) and off[-1].item() == 3
    assert np.array_equal(perm.cpu().numpy(), operm)


def test_permute_fp32_rows_bitwise():
    idx = cases.permute_indices(50, 4, 16, 0.0, seed=5)
    hidden = torch.randn(50, 96)
    p, _, _, perm = ek().moe_permute(hidden.cuda(), idx.cuda(), 16)
    assert torch.equal(p.cpu(), hidden[perm.cpu().long() // 4])


def test_permute_zero_tokens():
    p, off, s2d, perm = ek().moe_permute(torch.empty(0, 64, dtype=torch.bfloat16).cuda(),
                                         torch.empty(0, 8, dtype=torch.int32).cuda(), 16)
    assert p.shape == (0, 64) and off.shape == (17,) and int(off.abs().sum()) == 0


@pytest.mark.parametrize("T", [4096, 8192])
def test_permute_properties_full_size(T):
    """BASELINE cfg1 / cfg3 token counts at the DeepSeek-V3 row width:
    sorted, stable, inverse maps, offsets from counts, rows copied bitwise;
    then the round trip through the weighted unpermute with power-of-two
    weights summing to 1 (every fp32 partial sum exact) returns the tokens
    bit for bit."""
    from permute_props import check_permute_properties
    k, E, H = 8, 256, 7168
    idx = cases.permute_indices(T, k, E, 0.0, seed=T)
    g = torch.Generator(device="cuda").manual_seed(T)
    hidden = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    p, off, s2d, perm = ek().moe_permute(hidden, idx.cuda(), E)
    check_permute_properties(hidden, idx, E, p, off, s2d, perm)
    w = torch.tensor([0.5, 0.25, 0.125, 0.0625, 0.03125, 0.015625, 0.0078125, 0.0078125],
                     device="cuda").expand(T, k).contiguous()
    back = ek().moe_unpermute(p, w, s2d, T, k)
    assert torch.equal(back.view(torch.int16), hidden.view(torch.int16))


# ---- routing only (moe_route) ----------------------------------------------------

@pytest.mark.parametrize("name", ["t128_k4_e32", "t96_k8_e64_sentinels", "t1_k8_e256",
                                  "t4096_k8_e256"])
def test_route_golden(golden_dir, name):
    d = np.load(os.path.join(golden_dir, f"permute_{name}.npz"))
    import layerstormexpertkernels_b200 as P
    off, s2d, perm = P.moe_route(dev(d["topk_indices"]), int(d["num_experts"]))
    assert np.array_equal(perm.cpu().numpy(), d["perm"])
    assert np.array_equal(s2d.cpu().numpy(), d["s2d"])
    assert np.array_equal(off.cpu().numpy(), d["offsets"])


@pytest.mark.parametrize("T,k,E,sent", [
    (1, 1, 1, 0.0), (2, 8, 256, 0.0), (31, 3, 5, 0.2), (33, 8, 256, 0.0), (128, 8, 256, 0.0),
    (4096, 8, 256, 0.0), (4097, 8, 256, 0.05), (8192, 8, 256, 0.0), (20000, 6, 1023, 0.01),
    (3, 32, 64, 0.0), (1, 8, 1023, 0.5), (65536, 8, 256, 0.001), (4095, 8, 2, 0.0),
])
def test_route_vs_oracle(T, k, E, sent):
    """One launch, one CTA per two experts, every CTA reading all T*k keys:
    maps and offsets bit-exact against the oracle's stable sort, including
    sentinel keys, E = 1023 (512 CTAs), an odd expert count (the last CTA's
    second slot is past the sentinel bin), a key count that is not a multiple
    of 32, and 524288 keys (16 rounds of 32768 per CTA)."""
    import layerstormexpertkernels_b200 as P
    idx = cases.permute_indices(T, k, E, sent, seed=T * 7 + k)
    off, s2d, perm = P.moe_route(idx.cuda(), E)
    _, ooff, os2d, operm = O.moe_permute(None, idx.numpy(), E)
    assert np.array_equal(perm.cpu().numpy(), operm)
    assert np.array_equal(s2d.cpu().numpy(), os2d)
    assert np.array_equal(off.cpu().numpy(), ooff)


@pytest.mark.parametrize("T,k,E", [(37, 3, 16), (1000, 7, 256), (4099, 8, 1023)])
def test_route_arbitrary_invalid_keys(T, k, E):
    """Every id outside [0, E) is the sentinel bin, whatever its bit pattern
    (-1, -2, INT_MIN, INT_MAX, E, E + 1, ...), including in the last, partial
    16-byte vector of keys, where padding positions must stay out of it."""
    import layerstormexpertkernels_b200 as P
    g = torch.Generator().manual_seed(T + k)
    idx = torch.randint(-3, E + 3, (T, k), generator=g, dtype=torch.int32)
    flat = idx.view(-1)
    specials = torch.tensor([-2, -(2 ** 31), 2 ** 31 - 1, E, E + 1, -1, 0, E - 1],
                            dtype=torch.int32)
    flat[-len(specials):] = specials
    flat[: len(specials)] = specials
    off, s2d, perm = P.moe_route(idx.cuda(), E)
    _, ooff, os2d, operm = O.moe_permute(None, idx.numpy(), E)
    assert np.array_equal(perm.cpu().numpy(), operm)
    assert np.array_equal(s2d.cpu().numpy(), os2d)
    assert np.array_equal(off.cpu().numpy(), ooff)


def test_route_unaligned_indices_and_matches_permute():
    """topk_indices that start 4 bytes past a 16-byte boundary take the
    scalar key loads; the maps equal moe_permute's."""
    import layerstormexpertkernels_b200 as P
    idx = cases.permute_indices(3000, 8, 256, 0.01, seed=9)
    buf = torch.empty(3000 * 8 + 1, dtype=torch.int32, device="cuda")
    buf[1:] = idx.cuda().view(-1)
    view = buf[1:].view(3000, 8)
    assert view.data_ptr() % 16 != 0
    off, s2d, perm = P.moe_route(view, 256)
    hidden = rand_bf16((3000, 32), seed=2).cuda()
    _, poff, ps2d, pperm = ek().moe_permute(hidden, idx.cuda(), 256)
    assert torch.equal(off, poff) and torch.equal(s2d, ps2d) and torch.equal(perm, pperm)


def test_route_zero_tokens_and_rejections():
    import layerstormexpertkernels_b200 as P
    off, s2d, perm = P.moe_route(torch.empty(0, 8, dtype=torch.int32).cuda(), 16)
    torch.cuda.synchronize()
    assert off.shape == (17,) and int(off.abs().sum()) == 0 and s2d.numel() == 0
    with pytest.raises(RuntimeError):
        P.moe_route(torch.zeros(4, 8, dtype=torch.int32).cuda(), 1024)
    with pytest.raises(ValueError):
        P.moe_route(torch.zeros(4, 33, dtype=torch.int32).cuda(), 16)


def test_reference_roundtrip_case():
    # tests/test_kernels.py:58-88
    B, D, E, k = 128, 512, 32, 4
    tokens = torch.randn(B, D, dtype=torch.bfloat16, device="cuda")
    idx = torch.randint(0, E, (B, k), dtype=torch.int32, device="cuda")
    permuted, offsets, s2d, perm = ek().moe_permute(tokens, idx, E)
    assert permuted.shape == (B * k, D) and offsets.shape[0] == E + 1
    w = torch.full((B, k), 1.0 / k, dtype=torch.float32, device="cuda")
    rec = ek().moe_unpermute(permuted, w, s2d, B, k)
    assert (rec.float() - tokens.float()).abs().max().item() < 0.02


# ---- unpermute family --------------------------------------------------------------

def unpermute_inputs(T, k, H, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    permuted = (torch.randn(T * k, H, generator=g)).to(dtype)
    w = torch.rand(T, k, generator=g)
    s2d = torch.randperm(T * k, generator=g).int()
    return permuted, w, s2d


@pytest.mark.parametrize("T,k,H", [(1, 1, 8), (7, 8, 7168), (96, 8, 7168), (300, 6, 1000),
                                   (64, 3, 13), (5, 16, 256), (9, 32, 64), (1024, 8, 2048)])
def test_unpermute_sum_exact(T, k, H):
    permuted, w, s2d = unpermute_inputs(T, k, H, seed=T * k + H)
    out = ek().moe_unpermute(permuted.cuda(), w.cuda(), s2d.cuda(), T, k)
    ref = O.moe_unpermute(bits(permuted), w.numpy(), s2d.numpy(), T, k)
    assert np.array_equal(bits(out), ref)


def test_unpermute_sum_fp16_exact():
    permuted, w, s2d = unpermute_inputs(40, 8, 512, seed=9, dtype=torch.float16)
    out = ek().moe_unpermute(permuted.cuda(), w.cuda(), s2d.cuda(), 40, 8)
    assert out.dtype == torch.float16
    ref = O.moe_unpermute(bits(permuted), w.numpy(), s2d.numpy(), 40, 8, fp16=True)
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("T,k,H", [(96, 8, 7168), (5, 3, 13), (1, 8, 64)])
def test_perslot_and_reduce_exact(T, k, H):
    permuted, w, s2d = unpermute_inputs(T, k, H, seed=H + k)
    pc, wc, sc = permuted.cuda(), w.cuda(), s2d.cuda()
    x = permuted.float().numpy()
    f32 = ek().moe_unpermute_fp32(pc, wc, sc, T, k)
    of32 = O.moe_unpermute_perslot_f32(x, w.numpy(), s2d.numpy(), T, k)
    assert f32.dtype == torch.float32 and f32.shape == (T, k, H)
    assert np.array_equal(f32.cpu().numpy(), of32)
    b16 = ek().moe_unpermute_bf16_perslot(pc, wc, sc, T, k)
    ob16 = O.moe_unpermute_perslot_bf16(x, w.numpy(), s2d.numpy(), T, k)
    assert np.array_equal(bits(b16), O.bf16_bits(ob16))
    r32 = ek().moe_combine_reduce_slots_fp32_to_bf16(f32)
    assert np.array_equal(bits(r32), O.bf16_bits(O.reduce_slots(of32)))
    r16 = ek().moe_combine_reduce_slots_bf16_to_bf16(b16)
    assert np.array_equal(bits(r16), O.bf16_bits(O.reduce_slots(ob16)))


def test_reference_perslot_cases():
    # tests/test_kernels.py:90-200: per-slot outputs exact, reduce equals the
    # in-order fp32 sum, and split-invariance of the gathered slots.
    B, D, E, k = 96, 7168, 64, 8
    tokens = torch.randn(B, D, dtype=torch.bfloat16, device="cuda")
    idx = torch.randint(0, E, (B, k), dtype=torch.int32, device="cuda")
    permuted, _, s2d_map, _ = ek().moe_permute(tokens, idx, E)
    weights = torch.rand(B, k, dtype=torch.float32, device="cuda")
    s2d = s2d_map.view(B, k)
    per32 = ek().moe_unpermute_fp32(permuted, weights, s2d_map, B, k)
    ref = torch.zeros(B, k, D, device="cuda")
    for j in range(k):
        ref[:, j, :] = weights[:, j:j + 1] * permuted[s2d[:, j].long()].float()
    assert torch.equal(per32, ref)
    out = ek().moe_combine_reduce_slots_fp32_to_bf16(per32.contiguous())
    acc = torch.zeros(B, D, device="cuda")
    for j in range(k):
        acc += per32[:, j, :]
    assert torch.equal(out, acc.to(torch.bfloat16))
    for split in (1, 3, 5):
        a = per32.clone(); a[:, split:, :] = 0.0
        b = per32.clone(); b[:, :split, :] = 0.0
        assert torch.equal(ek().moe_combine_reduce_slots_fp32_to_bf16((a + b).contiguous()), out)
    per16 = ek().moe_unpermute_bf16_perslot(permuted, weights, s2d_map, B, k)
    ref16 = torch.zeros(B, k, D, dtype=torch.bfloat16, device="cuda")
    for j in range(k):
        ref16[:, j, :] = (weights[:, j:j + 1] * permuted[s2d[:, j].long()].float()).to(torch.bfloat16)
    assert torch.equal(per16, ref16)
    out16 = ek().moe_combine_reduce_slots_bf16_to_bf16(per16.contiguous())
    acc = torch.zeros(B, D, device="cuda")
    for j in range(k):
        acc += per16[:, j, :].float()
    assert torch.equal(out16, acc.to(torch.bfloat16))
    for split in (1, 3, 5):
        a = per16.clone(); a[:, split:, :] = 0.0
        b = per16.clone(); b[:, :split, :] = 0.0
        assert torch.equal(ek().moe_combine_reduce_slots_bf16_to_bf16((a + b).contiguous()), out16)


# ---- SwiGLU ----------------------------------------------------------------------------

def check_swiglu(out, gate, up, limit):
    ref = O.swiglu(gate.float().numpy(), up.float().numpy(), limit)
    got = out.float().cpu().numpy().astype(np.float64)
    # One rounding to the 16-bit format of a value within a few fp32 ulps of
    # the exact result: at most one 16-bit ulp away from it.  Below 2^-100
    # silu(g) flushes to 0 (the kernel's quotient once 1 + e^-g passes 2^126,
    # g < -87; fp32's e^-g itself for g < -88.7, as in the reference's torch
    # F.silu); the double-precision oracle keeps the tiny value, so those
    # elements only need to be tiny.
    if out.dtype == torch.bfloat16:
        ulp = np.maximum(np.abs(ref) * 2.0 ** -7, 2.0 ** -100)
    else:
        ulp = np.maximum(np.abs(ref) * 2.0 ** -10, 2.0 ** -24)
    assert (np.abs(got - ref) <= ulp).all(), np.abs(got - ref).max()


@pytest.mark.parametrize("N,d,limit,scale", [(256, 2048, 0.0, 1.0), (256, 2048, 10.0, 15.0),
                                             (1, 512, 0.0, 1.0), (33, 100, 0.0, 3.0),
                                             (4096, 2048, 0.0, 1.0), (7, 8, 10.0, 40.0)])
def test_swiglu_vs_oracle(N, d, limit, scale):
    gate = rand_bf16((N, d), seed=N + d, scale=scale)
    up = rand_bf16((N, d), seed=N * d, scale=scale)
    out = ek().fused_swiglu(torch.cat([gate, up], 1).cuda(), swiglu_limit=limit)
    check_swiglu(out.cpu(), gate, up, limit)


@pytest.mark.parametrize("name", ["plain", "clamp10", "edges"])
def test_swiglu_golden(golden_dir, name):
    # The reference's own ref_swiglu outputs (tests/golden/make_golden.py).
    d = np.load(os.path.join(golden_dir, f"swiglu_{name}.npz"))
    gate = torch.from_numpy(d["gate"]).to(torch.bfloat16)
    up = torch.from_numpy(d["up"]).to(torch.bfloat16)
    out = ek().fused_swiglu(torch.cat([gate, up], 1).cuda(), swiglu_limit=float(d["limit"]))
    got = out.float().cpu().numpy().astype(np.float64)
    ref = d["out"].astype(np.float64)
    assert (np.abs(got - ref) <= np.maximum(np.abs(ref) * 2.0 ** -7, 2.0 ** -100)).all()


def test_swiglu_full_size_sweep_shape():
    """BASELINE cfg2's largest call, [65536, 2*2048] bf16 ~ N(0,1): every output
    within one bf16 ulp of silu(g)*u evaluated in float64 on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(65536)
    x = torch.randn(65536, 4096, generator=g, device="cuda").to(torch.bfloat16)
    out = ek().fused_swiglu(x)
    gd, ud = x[:, :2048].double(), x[:, 2048:].double()
    ref = gd / (1.0 + torch.exp(-gd)) * ud
    tol = torch.clamp(ref.abs() * 2.0 ** -7, min=2.0 ** -100)
    assert bool(((out.double() - ref).abs() <= tol).all())


def test_swiglu_fp16():
    gate = rand_bf16((64, 256), seed=1, dtype=torch.float16)
    up = rand_bf16((64, 256), seed=2, dtype=torch.float16)
    out = ek().fused_swiglu(torch.cat([gate, up], 1).cuda())
    assert out.dtype == torch.float16
    check_swiglu(out.cpu(), gate, up, 0.0)


def test_reference_swiglu_cases():
    # tests/test_kernels.py:41-56, 318-336 and tests/test_fused_swiglu.py:127-201
    N, D = 256, 2048
    gate = torch.randn(N, D, dtype=torch.bfloat16, device="cuda")
    up = torch.randn(N, D, dtype=torch.bfloat16, device="cuda")
    out = ek().fused_swiglu(torch.cat([gate, up], 1))
    ref = F.silu(gate.float()) * up.float()
    assert F.cosine_similarity(out.float().flatten(), ref.flatten(), dim=0).item() > 0.9999
    assert torch.equal(out, ek().fused_swiglu(torch.cat([gate, up], 1), swiglu_limit=0.0))
    g20 = torch.randn(128, 1024, dtype=torch.bfloat16, device="cuda") * 20
    ones = torch.ones(128, 1024, dtype=torch.bfloat16, device="cuda")
    c = ek().fused_swiglu(torch.cat([g20, ones], 1), swiglu_limit=10.0)
    assert c.float().max().item() <= F.silu(torch.tensor(10.0)).item() + 0.05
    assert ek().fused_swiglu(torch.empty(0, 128, dtype=torch.bfloat16, device="cuda")).shape == (0, 64)
