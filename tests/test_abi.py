"""The C ABI boundary on the CPU: liblsek.so loads, exports exactly what
include/lsek.h declares, and rejects invalid arguments with the documented
status before any CUDA call (so these run without a GPU)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "lsek.h")
LIB = os.path.join(ROOT, "layerstormexpertkernels_b200", "liblsek.so")

LSEK_OK, LSEK_ERR_INVALID_ARG, LSEK_ERR_UNSUPPORTED = 0, 1, 2


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^LSEK_API\s+[\w\s\*]+?\b(lsek_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "liblsek.so not built (python layerstormexpertkernels_b200/build.py)"
    lib = ctypes.CDLL(LIB)
    lib.lsek_last_error.restype = ctypes.c_char_p
    lib.lsek_version.restype = ctypes.c_char_p
    return lib


class GatingParams(ctypes.Structure):
    _fields_ = [("num_tokens", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("topk", ctypes.c_int32), ("n_group", ctypes.c_int32),
                ("topk_group", ctypes.c_int32), ("routed_scaling_factor", ctypes.c_float),
                ("renormalize", ctypes.c_int32), ("scoring_func", ctypes.c_int32)]


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in ["lsek_topk_gating", "lsek_moe_permute", "lsek_moe_unpermute",
              "lsek_fused_swiglu", "lsek_grouped_gemm_bf16", "lsek_moe_layer_forward"]:
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in lsek.h but not exported"


def test_library_exports_nothing_else():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = sorted(line.split()[-1] for line in out.splitlines() if " T " in line)
    assert exported == declared_symbols()


def test_version(lib):
    assert lib.lsek_version().decode().startswith("lsek ")


def _gating(lib, **kw):
    p = GatingParams(num_tokens=4, num_experts=256, topk=8, n_group=8, topk_group=4,
                     routed_scaling_factor=2.5, renormalize=1, scoring_func=0)
    for k, v in kw.items():
        setattr(p, k, v)
    dummy = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    return lib.lsek_topk_gating(dummy, dummy, dummy, None, ctypes.byref(p), None)


@pytest.mark.parametrize("kw,needle", [
    (dict(num_experts=0), "num_experts"),
    (dict(topk=0), "topk"),
    (dict(topk=300), "topk"),
    (dict(n_group=7), "divisible"),
    (dict(topk_group=9), "topk_group"),
    (dict(topk_group=0), "topk_group"),
    (dict(topk=140, topk_group=4), "kept groups"),
    (dict(scoring_func=5), "scoring_func"),
    (dict(num_tokens=-1), "num_tokens"),
])
def test_gating_invalid_args(lib, kw, needle):
    assert _gating(lib, **kw) == LSEK_ERR_INVALID_ARG
    assert needle in lib.lsek_last_error().decode()


def test_gating_unsupported_sizes(lib):
    assert _gating(lib, num_experts=2048, n_group=1, topk_group=1) == LSEK_ERR_UNSUPPORTED


def test_gating_zero_tokens_is_noop(lib):
    assert _gating(lib, num_tokens=0) == LSEK_OK


def test_permute_invalid_args(lib):
    d = ctypes.c_void_p(16)
    st = lib.lsek_moe_permute(d, d, d, d, d, d, 4, 8, 64, 256, 3, None, ctypes.c_size_t(0), None)
    assert st == LSEK_ERR_INVALID_ARG and b"elem_size_bytes" in lib.lsek_last_error()
    st = lib.lsek_moe_permute(d, d, d, d, d, d, 4, 8, 64, 4096, 2, None, ctypes.c_size_t(0), None)
    assert st == LSEK_ERR_UNSUPPORTED


def test_route_invalid_args(lib):
    d = ctypes.c_void_p(16)
    assert lib.lsek_moe_route(d, d, d, d, 4, 33, 256, None) == LSEK_ERR_INVALID_ARG
    assert b"topk" in lib.lsek_last_error()
    assert lib.lsek_moe_route(d, d, d, d, -1, 8, 256, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_moe_route(d, d, d, d, 4, 8, 0, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_moe_route(None, d, d, d, 4, 8, 256, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_moe_route(d, None, d, d, 4, 8, 256, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_moe_route(d, d, d, d, 4, 8, 1024, None) == LSEK_ERR_UNSUPPORTED


def test_noalloc_permute_size_limit(lib):
    """The static-buffer permute rejects, before touching the GPU, the first
    size past its 1 MiB of route counts: at E=256 that is one slot past
    2,088,960 (1021 chunks of 2048 slots x 257 counts x 4 bytes)."""
    d = ctypes.c_void_p(256)
    limit = 1 << 20  # LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES
    assert ((2_088_960 + 2047) // 2048) * 257 * 4 <= limit
    assert ((2_088_961 + 2047) // 2048) * 257 * 4 > limit
    st = lib.lsek_moe_permute_noalloc(d, d, d, d, d, d, 2_088_961, 1, 8, 256, 2, None)
    assert st == LSEK_ERR_INVALID_ARG and b"static buffer" in lib.lsek_last_error()
    st = lib.lsek_moe_permute_noalloc(d, d, d, d, d, d, 261121, 8, 8, 256, 2, None)
    assert st == LSEK_ERR_INVALID_ARG and b"static buffer" in lib.lsek_last_error()


def test_unpermute_topk_limit(lib):
    d = ctypes.c_void_p(16)
    st = lib.lsek_moe_unpermute(d, d, d, d, 4, 33, 64, 0, 0, None)
    assert st == LSEK_ERR_INVALID_ARG and b"topk" in lib.lsek_last_error()


def test_swiglu_invalid(lib):
    d = ctypes.c_void_p(16)
    assert lib.lsek_fused_swiglu(d, d, 4, 8, ctypes.c_float(-1.0), 0, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_fused_swiglu(d, d, 4, 8, ctypes.c_float(0.0), 2, None) == LSEK_ERR_INVALID_ARG


def test_gemm_invalid(lib):
    d = ctypes.c_void_p(16)
    z = ctypes.c_size_t(0)
    assert lib.lsek_grouped_gemm_bf16(d, d, d, d, 4, 8, 64, 12, None, z, None) == LSEK_ERR_INVALID_ARG  # K % 8
    assert lib.lsek_grouped_gemm_bf16(d, d, d, d, 4, 8, 48, 64, None, z, None) == LSEK_ERR_INVALID_ARG  # N % 32
    assert lib.lsek_grouped_gemm_bf16(d, d, d, d, 2048, 8, 64, 64, None, z, None) == LSEK_ERR_UNSUPPORTED
    odd = ctypes.c_void_p(18)
    assert lib.lsek_grouped_gemm_bf16(d, odd, d, d, 4, 8, 64, 64, None, z, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_grouped_gemm_bf16(d, d, d, d, 4, 8, 64, 0, None, z, None) == LSEK_ERR_INVALID_ARG  # K = 0
    assert b"K must be > 0" in lib.lsek_last_error()


def test_adaptive_invalid(lib):
    d = ctypes.c_void_p(16)
    f = lib.lsek_adaptive_gating
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                          ctypes.c_void_p]
    assert f(d, d, d, d, d, 4, 0, 0.5, None) == LSEK_ERR_INVALID_ARG
    assert f(d, d, d, d, d, 4, 8, 1.5, None) == LSEK_ERR_INVALID_ARG


def test_workspace_sizes(lib):
    lib.lsek_moe_permute_workspace_size.restype = ctypes.c_size_t
    lib.lsek_moe_layer_workspace_size.restype = ctypes.c_size_t
    small = lib.lsek_moe_permute_workspace_size(128, 8, 256)
    big = lib.lsek_moe_permute_workspace_size(65536, 8, 256)
    assert small > 0 and big > small and big % 256 == 0
    ws = lib.lsek_moe_layer_workspace_size(4096, 7168, 2048, 256, 8)
    # at least X [T*k,H] + Hact [T*k,I] in bf16
    assert ws >= 4096 * 8 * (7168 + 2048) * 2


def test_ep_entry_points_reject_bad_arguments(lib):
    """The expert-parallel entry points validate before any CUDA call."""
    d = ctypes.c_void_p(16)
    z = ctypes.c_size_t(0)
    f = lib.lsek_ep_plan
    # world size 0, experts not a multiple of the world size, topk out of range
    assert f(d, d, d, d, d, 4, 8, 64, 0, d, z, None) == LSEK_ERR_INVALID_ARG
    assert f(d, d, d, d, d, 4, 8, 60, 8, d, z, None) == LSEK_ERR_INVALID_ARG
    assert f(d, d, d, d, d, 4, 33, 64, 8, d, z, None) == LSEK_ERR_INVALID_ARG
    assert f(d, d, d, d, d, 4, 8, 64, 65, d, z, None) == LSEK_ERR_INVALID_ARG
    # hidden_dim must be a multiple of 8
    g = lib.lsek_ep_dispatch_pack
    assert g(d, d, d, 4, d, d, d, d, d, 4, 8, 12, 64, 8, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_ep_slot_scan(d, d, -1, 8, None) == LSEK_ERR_INVALID_ARG
    h = lib.lsek_ep_expert_permute
    assert h(d, 4, d, d, d, d, d, 4, 8, 64, 0, d, z, None) == LSEK_ERR_INVALID_ARG  # 0 local experts
    assert lib.lsek_ep_combine_pack(d, -1, d, d, d, d, d, 4, 8, 64, None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_ep_combine_reduce(d, d, -1, d, d, d, 4, 8, 64, 64, 8, None) == LSEK_ERR_INVALID_ARG


def test_ep_domain_entry_points_reject_bad_arguments(lib):
    out = ctypes.c_void_p()
    create = lib.lsek_ep_domain_create
    assert create(ctypes.byref(out), 0, 17, 64, 64, 8) == LSEK_ERR_INVALID_ARG   # world > 16
    assert create(ctypes.byref(out), 2, 2, 64, 64, 8) == LSEK_ERR_INVALID_ARG    # rank >= world
    assert create(ctypes.byref(out), 0, 2, 64, 60, 8) == LSEK_ERR_INVALID_ARG    # H % 8
    assert create(ctypes.byref(out), 0, 2, 0, 64, 8) == LSEK_ERR_INVALID_ARG     # no tokens
    assert out.value is None
    assert lib.lsek_ep_domain_export(None, ctypes.c_void_p(16), ctypes.c_size_t(64)) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_ep_wait(None, 0, 1, 0, None) == LSEK_ERR_INVALID_ARG
    d = ctypes.c_void_p(16)
    assert lib.lsek_ep_combine_plan_chunks(None, d, d, d, d, d, d, d, d, 4, 4, 16, 4,
                                           None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_ep_combine_plan_chunks(None, d, d, d, d, d, d, d, d, 4, 4, 16, 0,
                                           None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_ep_combine_push_chunk(None, d, d, d, d, 4, None, None, d, d, 0, 1,
                                          None) == LSEK_ERR_INVALID_ARG
    lib.lsek_ep_domain_bytes.restype = ctypes.c_size_t
    one = lib.lsek_ep_domain_bytes(8192, 7168, 8, 8)
    # control block + recv rows [T*G, H] + ids / weights [T*G, k] + source tokens [T*G]
    # + combine rows [T*k, H]
    assert one >= (16384 + 8192 * 8 * 7168 * 2 + 2 * 8192 * 8 * 8 * 4 + 8192 * 8 * 4
                   + 8192 * 8 * 7168 * 2)
    assert lib.lsek_ep_domain_bytes(-1, 7168, 8, 8) == 0
    lib.lsek_ep_domain_destroy(None)  # a no-op


def test_copy_to_mapped_host_rejects_bad_arguments(lib):
    # All of these return before any CUDA call.
    d = ctypes.c_void_p(16)
    assert lib.lsek_copy_to_mapped_host(d, d, ctypes.c_size_t(6), None) == LSEK_ERR_INVALID_ARG
    assert b"multiple of 4" in lib.lsek_last_error()
    assert lib.lsek_copy_to_mapped_host(None, d, ctypes.c_size_t(8), None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_copy_to_mapped_host(d, ctypes.c_void_p(18), ctypes.c_size_t(8),
                                        None) == LSEK_ERR_INVALID_ARG
    assert lib.lsek_copy_to_mapped_host(None, None, ctypes.c_size_t(0), None) == 0
