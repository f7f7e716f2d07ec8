"""GPU parity of the tcgen05 grouped GEMM (plain and with the SwiGLU
epilogue) against the oracle's double-precision contraction.  Bar (north
star): bf16 outputs within rtol 2e-2 / atol 1e-2 of the fp32-accumulated
reference; the fused SwiGLU epilogue bit-identical to GEMM + fused_swiglu."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_util import assert_close_bf16, sync_and_check_device_error
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def ek():
    import sm120_expert_kernels as EK
    return EK


def make_problem(counts, K, N, seed, wscale=0.05, pad_rows=0):
    g = torch.Generator().manual_seed(seed)
    rows = int(sum(counts)) + pad_rows
    a = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(len(counts), N, K, generator=g) * wscale).to(torch.bfloat16)
    offsets = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
    return a, b, offsets


def oracle_gemm(a, b, offsets):
    return O.grouped_gemm(a.float().numpy(), b.float().numpy(), offsets.numpy())


def test_reference_golden_case(golden_dir):
    d = np.load(os.path.join(golden_dir, "grouped_gemm_e4.npz"))
    a = torch.as_tensor(d["a"]).to(torch.bfloat16).cuda()
    b = torch.as_tensor(d["b"]).to(torch.bfloat16).cuda()
    out = ek().grouped_gemm_bf16(a, b, torch.as_tensor(d["offsets"]).cuda())
    sync_and_check_device_error()
    assert_close_bf16(out, d["out"])


@pytest.mark.parametrize("counts,K,N", [
    ([1], 64, 256),
    ([128], 64, 256),
    ([129, 0, 1, 255, 256, 300], 256, 256),
    ([17, 33, 0, 64], 72, 96),          # K tail (72 = 64 + 8), N not a multiple of 256
    ([200, 50], 1024, 320),
    ([40] * 16, 7168, 256),
    ([130, 3, 0, 0, 77], 2048, 7168),
])
def test_grouped_gemm_vs_oracle(counts, K, N):
    a, b, off = make_problem(counts, K, N, seed=K + N + len(counts))
    out = ek().grouped_gemm_bf16(a.cuda(), b.cuda(), off.cuda())
    sync_and_check_device_error()
    assert_close_bf16(out, oracle_gemm(a, b, off))


def test_grouped_gemm_tight_error():
    # Beyond the bar: an fp32-accumulated result rounded once to bf16 is at
    # most ~1 bf16 ulp from the exact value.
    a, b, off = make_problem([256, 100, 31], 2048, 512, seed=7)
    out = ek().grouped_gemm_bf16(a.cuda(), b.cuda(), off.cuda()).float().cpu().numpy()
    ref = oracle_gemm(a, b, off)
    err = np.abs(out - ref) / np.maximum(np.abs(ref), 1e-3)
    assert np.quantile(err, 0.999) <= 2 ** -7 and err.max() <= 2 ** -5


def test_rows_outside_experts_untouched():
    """Rows past offsets[E] (adaptive-gating sentinels) are not written; the
    C ABI is driven directly so the output buffer can carry a canary."""
    import layerstormexpertkernels_b200 as P
    a, b, off = make_problem([30, 0, 50], 128, 64, seed=3, pad_rows=20)
    a, b, off = a.cuda(), b.cuda(), off.cuda()
    d = torch.full((a.shape[0], 64), 7.0, dtype=torch.bfloat16, device="cuda")
    lib = ctypes.CDLL(P.LIBRARY_PATH)
    st = lib.lsek_grouped_gemm_bf16(
        ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
        ctypes.c_void_p(off.data_ptr()), 3, a.shape[0], 64, 128, None, ctypes.c_size_t(0),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    sync_and_check_device_error()
    assert (d[80:] == 7.0).all()
    assert_close_bf16(d[:80], oracle_gemm(a.cpu(), b.cpu(), off.cpu())[:80])


@pytest.mark.parametrize("counts,K,I,limit", [
    ([5, 128, 0, 200], 256, 128, 0.0),
    ([64, 64], 7168, 256, 0.0),
    ([300, 1], 512, 2048, 10.0),
    ([33], 64, 96, 0.0),
])
def test_swiglu_epilogue_equals_unfused(counts, K, I, limit):
    # Weights scaled so g, u ~ N(0, 1) (x4 when the clamp is exercised): the
    # output bar is relative to h, while a one-ulp difference in the bf16
    # rounding of g or u moves h by silu(g) * ulp(u).
    wscale = (4.0 if limit > 0 else 1.0) / np.sqrt(K)
    a, w, off = make_problem(counts, K, 2 * I, seed=K + I, wscale=wscale)
    a, w, off = a.cuda(), w.cuda(), off.cuda()
    fused = ek().grouped_gemm_swiglu_bf16(a, w, off, swiglu_limit=limit)
    gu = ek().grouped_gemm_bf16(a, w, off)
    unfused = ek().fused_swiglu(gu, swiglu_limit=limit)
    sync_and_check_device_error()
    assert torch.equal(fused, unfused)
    gu_ref = O.bf16_round(oracle_gemm(a.cpu(), w.cpu(), off.cpu()).astype(np.float32))
    ref = O.swiglu(gu_ref[:, :I], gu_ref[:, I:], limit)
    assert_close_bf16(fused, ref)


def test_deepseek_shape_subset():
    """Eight experts of the DeepSeek-V3 layer (H=7168, I=2048) with ~128 rows
    each: gate/up + SwiGLU then down, against the double-precision oracle."""
    from layerstormexpertkernels_b200.synthetic import expert_weights
    w_gu, w_down = expert_weights(8, 7168, 2048, device="cuda")
    counts = [128, 97, 160, 128, 1, 250, 128, 130]
    g = torch.Generator().manual_seed(11)
    x = torch.randn(sum(counts), 7168, generator=g).to(torch.bfloat16)
    off = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
    h = ek().grouped_gemm_swiglu_bf16(x.cuda(), w_gu, off.cuda())
    y = ek().grouped_gemm_bf16(h, w_down, off.cuda())
    sync_and_check_device_error()
    xs = x.float().numpy()
    for e in range(8):
        s, t = int(off[e]), int(off[e + 1])
        ref = O.expert_ffn(xs[s:t], w_gu[e].float().cpu().numpy(), w_down[e].float().cpu().numpy())
        assert_close_bf16(y[s:t], ref)


def test_empty_problem():
    a = torch.empty(0, 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(3, 64, 64, dtype=torch.bfloat16, device="cuda")
    off = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert ek().grouped_gemm_bf16(a, b, off).shape == (0, 64)


@pytest.mark.parametrize("swiglu", [False, True])
def test_tile_shape_does_not_change_results(swiglu):
    """A row's output must not depend on how many other rows share its
    expert: calls of at most 32 rows run the decode geometry (swapped MMA
    operands, weights on M), larger ones unswapped tiles, and both must give
    the same bits.  Expert parallelism
    relies on this (an expert's rows are grouped differently on each rank)."""
    K, N = 1024, 512
    g = torch.Generator().manual_seed(99)
    a = torch.randn(128, K, generator=g).to(torch.bfloat16).cuda()
    b = (torch.randn(1, N, K, generator=g) / np.sqrt(K)).to(torch.bfloat16).cuda()

    def run(rows):
        off = torch.tensor([0, rows], dtype=torch.int32, device="cuda")
        if swiglu:
            return ek().grouped_gemm_swiglu_bf16(a[:rows].contiguous(), b, off)
        return ek().grouped_gemm_bf16(a[:rows].contiguous(), b, off)

    full = run(128)
    for r in (1, 15, 16, 40, 64, 65, 100):
        assert torch.equal(run(r), full[:r]), f"rows={r}"
    sync_and_check_device_error()


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("K", [64, 576, 1024])
def test_paired_tiles_match_single_tiles(swiglu, K):
    """Experts with more than 128 rows run as paired units (two
    accumulators against one weight tile, up to 256 rows), wide swapped
    tiles of 129..192 rows (N up to 192), and, when at most 64 rows follow a
    256-row block, a full tile and a wide tile in place of that block; the
    rows must come out bit-identical to the same rows computed one 128-row
    tile per expert.  The k-block counts (1, 9, 16) move the shared-memory
    ring's wrap point through every box position."""
    N = 512
    g = torch.Generator().manual_seed(K + swiglu)
    b = (torch.randn(1, N, K, generator=g) / np.sqrt(K)).to(torch.bfloat16).cuda()
    for rows in (129, 192, 193, 200, 255, 256, 257, 300, 320, 321, 384, 400, 448, 449, 511,
                 520, 577):
        a = torch.randn(rows, K, generator=g).to(torch.bfloat16).cuda()
        off = torch.tensor([0, rows], dtype=torch.int32, device="cuda")
        cuts = list(range(0, rows, 128)) + [rows]
        split = torch.tensor(cuts, dtype=torch.int32, device="cuda")
        bs = b.expand(len(cuts) - 1, N, K).contiguous()
        if swiglu:
            whole = ek().grouped_gemm_swiglu_bf16(a, b, off)
            tiled = ek().grouped_gemm_swiglu_bf16(a, bs, split)
        else:
            whole = ek().grouped_gemm_bf16(a, b, off)
            tiled = ek().grouped_gemm_bf16(a, bs, split)
        sync_and_check_device_error()
        assert torch.equal(whole, tiled), f"rows={rows}"


def test_tail_tiles_of_large_experts():
    # Experts with 129..192 rows: one wide swapped tile each.
    a, b, off = make_problem([130, 192, 150, 129], 512, 256, seed=21)
    out = ek().grouped_gemm_bf16(a.cuda(), b.cuda(), off.cuda())
    sync_and_check_device_error()
    assert_close_bf16(out, oracle_gemm(a, b, off))


def test_decode_down_projection_matches_full_geometry():
    """A decode-sized down projection (at most 32 rows over a few experts,
    N = 7168) runs the decode geometry; its rows must equal the same rows
    computed by a full-geometry call, and the oracle."""
    K, N = 2048, 7168
    counts = [3, 0, 5, 1]
    a, b, off = make_problem(counts + [40], K, N, seed=5, wscale=1.0 / np.sqrt(K))
    a, b = a.cuda(), b.cuda()
    small_off = off[:len(counts) + 1].cuda()
    rows = int(sum(counts))
    small = ek().grouped_gemm_bf16(a[:rows].contiguous(), b[:len(counts)].contiguous(), small_off)
    full = ek().grouped_gemm_bf16(a, b, off.cuda())
    sync_and_check_device_error()
    assert torch.equal(small, full[:rows])
    assert_close_bf16(small, oracle_gemm(a[:rows].cpu(), b[:len(counts)].cpu(),
                                         off[:len(counts) + 1]))
