"""Host-side pieces of bench.py that need no GPU: the roofline bound choice
and the clock-sample summary."""
from __future__ import annotations

import bench

PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0,
         "source": "measured"}


def test_roofline_picks_hbm_for_weight_streaming():
    # cfg1 gate/up: 1.92 TFLOP over 15.6 GB -> the HBM floor (2.4 ms) is higher.
    r = bench.gemm_roofline("gu", 1.924e12, 15.64e9, 2.8, PEAKS)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert abs(r["achieved"] - 15.64e9 / 2.8e-3 / 1e9) < 1e-6
    assert abs(r["frac"] - r["achieved"] / PEAKS["hbm_gbs"]) < 1e-12


def test_roofline_picks_tensor_for_many_rows_per_expert():
    # An expert-parallel rank at 8 GPUs: 1024 rows per expert, 2.5 GB.
    r = bench.gemm_roofline("gu", 1.924e12, 2.51e9, 1.6, PEAKS)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - 1.924e12 / 1.6e-3 / 1e12) < 1e-6
    assert r["peak"] == PEAKS["bf16_tflops_sustained"]


def test_clock_summary_flags_throttle_reasons():
    s = bench.ClockSampler(0)
    s.samples = [(1965.0, 1965.0, frozenset({"sw_power_cap"})), (1800.0, 1965.0, frozenset())]
    out = s.summary()
    assert out["sm_mhz"] == (1965 + 1800) / 2 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 2


def test_bind_host_to_device_without_gpu_changes_nothing():
    import os

    import torch

    import layerstormexpertkernels_b200 as P
    if torch.cuda.is_available():
        return  # the GPU tests exercise it
    before = os.sched_getaffinity(0)
    assert P.bind_host_to_device(None) is None
    assert os.sched_getaffinity(0) == before
