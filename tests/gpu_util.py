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
