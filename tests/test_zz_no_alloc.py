"""The allocation-free permute entry point, lsek_moe_permute_noalloc.

Some callers of this library cannot allocate device memory around a call:
for instance a plugin host that is handed its input and output buffers by
another runtime and owns no allocator, or a runtime that plans all of its
device memory at start-up and treats any later cudaMalloc as an error.  For
them the permute keeps its scratch (the per-chunk expert counts of the
multi-CTA route) in a fixed 1 MiB device buffer inside liblsek instead of a
caller workspace.

The test drives the entry point through the C ABI and checks that it
produces exactly what lsek_moe_permute produces with a workspace, on two
calls in a row with different sizes, so the second call runs on the buffer
contents the first one left behind.  Both sizes are above the single-CTA
limit, so the scratch is in use.  The file is named to be collected last: a
run that stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LSEK_ERR_INVALID_ARG = 1


def load_lib():
    import layerstormexpertkernels_b200 as P
    lib = ctypes.CDLL(P.LIBRARY_PATH)
    lib.lsek_last_error.restype = ctypes.c_char_p
    lib.lsek_moe_permute_workspace_size.restype = ctypes.c_size_t
    return lib


def ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def run_permute(lib, hidden, idx, num_experts, noalloc: bool):
    T, H = hidden.shape
    k = idx.shape[1]
    dev = hidden.device
    permuted = torch.empty(T * k, H, dtype=hidden.dtype, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    s2d = torch.empty(T * k, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ptr(permuted), ptr(offsets), ptr(s2d), ptr(perm), ptr(hidden), ptr(idx), T, k, H,
            num_experts, hidden.element_size()]
    if noalloc:
        st = lib.lsek_moe_permute_noalloc(*args, stream)
    else:
        nbytes = lib.lsek_moe_permute_workspace_size(T, k, num_experts)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        st = lib.lsek_moe_permute(*args, ptr(ws), ctypes.c_size_t(nbytes), stream)
    assert st == 0, lib.lsek_last_error().decode()
    torch.cuda.synchronize()
    return permuted, offsets, s2d, perm


def test_noalloc_permute_matches_workspace_permute_on_two_calls():
    lib = load_lib()
    for T, k, E, H, seed in [(8192, 8, 256, 64, 1), (5000, 8, 128, 256, 2)]:
        g = torch.Generator().manual_seed(seed)
        idx = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32)
        idx[::13, 3] = -1  # adaptive-gating sentinels
        hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
        idx = idx.cuda()
        got = run_permute(lib, hidden, idx, E, noalloc=True)
        want = run_permute(lib, hidden, idx, E, noalloc=False)
        for name, a, b in zip(("permuted", "offsets", "src_to_dest", "permuted_idx"), got, want):
            assert torch.equal(a, b), f"{name} differs at T={T}, E={E}"


def test_noalloc_permute_at_its_largest_size():
    """The largest request the static buffer holds at E=256: 261120 tokens at
    top-8 (2,088,960 slots = 1020 route chunks of 2048, times 257 counts of
    4 bytes = exactly 1 MiB).  Bits equal the workspace permute's."""
    lib = load_lib()
    T, k, E, H = 261120, 8, 256, 8
    g = torch.Generator().manual_seed(3)
    idx = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32).cuda()
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    got = run_permute(lib, hidden, idx, E, noalloc=True)
    want = run_permute(lib, hidden, idx, E, noalloc=False)
    for name, a, b in zip(("permuted", "offsets", "src_to_dest", "permuted_idx"), got, want):
        assert torch.equal(a, b), f"{name} differs at the largest size"


def test_noalloc_permute_rejects_sizes_beyond_its_buffer():
    lib = load_lib()
    d = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    st = lib.lsek_moe_permute_noalloc(d, d, d, d, d, d, 1 << 20, 8, 64, 1023, 2, None)
    assert st == LSEK_ERR_INVALID_ARG
    assert b"static buffer" in lib.lsek_last_error()
