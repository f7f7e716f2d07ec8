"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    """16-bit tensor -> uint16 numpy bit patterns (host)."""
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def dev(x, dtype=None) -> torch.Tensor:
    t = torch.as_tensor(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def bf16_dev(x) -> torch.Tensor:
    """fp32 numpy values (exactly representable in bf16) -> bf16 CUDA tensor."""
    return torch.as_tensor(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).cuda()


def assert_close_bf16(got: torch.Tensor, ref: np.ndarray, rtol=2e-2, atol=1e-2):
    """The bf16 output bar: |got - ref| <= atol + rtol * |ref|."""
    g = f32(got).astype(np.float64)
    r = np.asarray(ref, dtype=np.float64)
    err = np.abs(g - r) - (atol + rtol * np.abs(r))
    worst = int(np.argmax(err)) if err.size else 0
    assert err.size == 0 or err.max() <= 0, (
        f"max excess {err.max():.3e} at flat index {worst}: got {g.flat[worst]}, ref {r.flat[worst]}")


def sync_and_check_device_error():
    import layerstormexpertkernels_b200 as P
    torch.cuda.synchronize()
    code = P.device_error()
    assert code == 0, f"kernel reported device error {code}"


def assert_layer_close(got: torch.Tensor, ref: np.ndarray, rtol=2e-2, atol=1e-2,
                       frac=0.999, slack=2.0, min_cos=0.9999):
    """End-to-end bar for the composed layer.  The GPU accumulates each GEMM
    in fp32 on the tensor cores, the oracle in double; each side rounds g, u,
    h and y to bf16, and where the two sit on opposite sides of a bf16
    rounding boundary the one-ulp differences propagate through the next
    contraction.  Every stage is checked on its own with the strict bar in
    test_gpu_gemm.py / test_gpu_permute.py; for the whole layer at least
    `frac` of the elements must meet |got - ref| <= atol + rtol*|ref|, all
    must meet it within `slack` times, and the cosine similarity must exceed
    `min_cos` (the reference's own layer-level criterion)."""
    g = f32(got).astype(np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    bound = atol + rtol * np.abs(r)
    err = np.abs(g - r)
    ok = float((err <= bound).mean())
    worst = int(np.argmax(err / bound))
    assert ok >= frac, f"only {ok:.5f} of elements within the bar"
    assert (err <= slack * bound).all(), (
        f"element {worst}: got {g[worst]}, ref {r[worst]} exceeds {slack}x the bar")
    cos = float(np.dot(g, r) / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-30))
    assert cos > min_cos, cos
