#!/usr/bin/env python
"""Benchmark: DeepSeek-V3 routed MoE layer forward on B200.

Workload ("cfg1"): T=4096 tokens per GPU, hidden 7168,
256 routed experts, moe_intermediate 2048, bf16 weights ~ N(0, 0.02), top-8
sigmoid routing with 8 groups / 4 kept, renormalised x2.5.  One step =
gating -> permute -> gate/up GEMM + SwiGLU -> down GEMM -> weighted unpermute
on one batch of synthetic tokens (seeded randn, no dataset).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is whole-job tokens/s with inputs resident in HBM, timed with CUDA
events over exactly K steps between barriers, max over ranks.  `e2e` is the
same metric through the public MoELayer call fed by HostPipeline from pinned
host buffers: each step copies hidden + logits host->device and the layer
output device->host, the copies overlapped with the neighbouring steps'
compute on their own streams.
The 22.5 GB of expert weights streamed every step exceed the 126 MB L2, so no
flush is needed.  `--impl reference` times the CPU restatement of the
reference's torch path (the oracle port) on the host cores.

With N > 1 (or --ep) the layer runs expert-parallel: each rank holds 4096
tokens and E/N experts, tokens travel to their experts' ranks and back with
NCCL all-to-alls (weak scaling in tokens; the experts are sharded).  The same
line then carries "ep_combine": the BASELINE configs[3] dispatch + weighted
combine (T=8192 tokens per rank, synthetic bf16 expert outputs) with its
off-rank bytes and GB/s per GPU against the NVLink peer-copy figure.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

T_TOKENS, HIDDEN, INTER, EXPERTS, TOPK, N_GROUP, TOPK_GROUP, RSF = 4096, 7168, 2048, 256, 8, 8, 4, 2.5
METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"
WORKLOAD = ("cfg1: DeepSeek-V3 routed MoE layer forward (gating, permute, gate/up GEMM + "
            "SwiGLU, down GEMM, weighted unpermute), T=4096 tokens/GPU, H=7168, I=2048, "
            "E=256, top-8, 8 groups / 4 kept, bf16 weights")
STAGES = ("gating", "route", "row_copy", "gate_up_swiglu_gemm", "down_gemm", "unpermute")


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """SM clock and throttle-reason samples of one GPU while running: NVML
    polled every 10 ms from a thread (a timed region of a few tens of
    milliseconds still gets samples), else `nvidia-smi -lms 200`.  The GPU is
    found by the PCI bus id of the torch device, so CUDA_VISIBLE_DEVICES
    renumbering does not matter."""

    # NVML clocks-event reason bits and the names the report uses.
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    SMI_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples = []  # (sm_mhz, max_mhz, frozenset of reason names)
        self.proc = None
        self.thread = None
        self.stop_flag = threading.Event()

    def _bus_id(self):
        import torch
        p = torch.cuda.get_device_properties(self.device_index)
        return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(self._bus_id())
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: nvidia-smi at its shortest interval
            self._start_smi()
            return

        def poll():
            while not self.stop_flag.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                    bits = get_reasons(handle)
                except Exception:
                    break
                self.samples.append((float(sm), float(max_mhz), frozenset(
                    n for n, b in self.REASON_BITS.items() if bits & b)))
                self.stop_flag.wait(0.01)
            pynvml.nvmlShutdown()

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def _start_smi(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--id=" + self._bus_id(), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 6 and parts[0].replace(".", "").isdigit():
                    self.samples.append((float(parts[0]), float(parts[1]) if parts[1].replace(
                        ".", "").isdigit() else 0.0, frozenset(
                        n for n, v in zip(self.SMI_REASONS, parts[2:6]) if v.lower() == "active")))

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        sm = [x[0] for x in self.samples]
        mx = [x[1] for x in self.samples if x[1] > 0]
        reasons = set()
        for x in self.samples:
            reasons |= x[2]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference's torch path
# ---------------------------------------------------------------------------

# Both CPU legs (the reference arm and the cpu_baseline of our arm) time the
# expert FFN on the same experts: CPU_SAMPLE_EXPERTS experts drawn with
# CPU_SAMPLE_SEED from the non-empty ones.
CPU_SAMPLE_EXPERTS = 4
CPU_SAMPLE_SEED = 0


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_layer_sample(logits, bias, hidden_bf16_f32, n_experts_sample=CPU_SAMPLE_EXPERTS,
                     seed=CPU_SAMPLE_SEED):
    """Times the CPU restatement of the layer on a bounded sample: gating,
    permute and unpermute over all tokens, the expert FFN on the rows of
    `n_experts_sample` experts, scaled by rows to all experts.  Returns a
    dict: est_s (estimated seconds for the full layer), the measured parts
    and the sample's size."""
    from oracle import moe_oracle as O
    t0 = time.perf_counter()
    w, idx = O.topk_gating(logits, bias, TOPK, N_GROUP, TOPK_GROUP, RSF, True)
    t1 = time.perf_counter()
    permuted, offsets, s2d, _ = O.moe_permute(hidden_bf16_f32, idx, EXPERTS)
    t2 = time.perf_counter()
    rng = np.random.default_rng(seed)
    counts = np.diff(offsets)
    experts = sorted(int(e) for e in rng.choice(np.nonzero(counts)[0], size=n_experts_sample,
                                                replace=False))
    y = np.zeros(permuted.shape, dtype=np.uint16)
    ffn = 0.0
    rows = 0
    for j, e in enumerate(experts):
        g = np.random.default_rng(1000 + int(e))
        w_gu = O.bf16_round((g.standard_normal((2 * INTER, HIDDEN), dtype=np.float32) * 0.02))
        w_dn = O.bf16_round((g.standard_normal((HIDDEN, INTER), dtype=np.float32) * 0.02))
        s, t = int(offsets[e]), int(offsets[e + 1])
        if j == 0:  # first BLAS call of the process: thread-pool start-up, untimed
            O.expert_ffn(permuted[s:s + 1], w_gu, w_dn, gemm_dtype=np.float32)
        f0 = time.perf_counter()
        y[s:t] = O.bf16_bits(O.expert_ffn(permuted[s:t], w_gu, w_dn, gemm_dtype=np.float32))
        ffn += time.perf_counter() - f0
        rows += t - s
    t3 = time.perf_counter()
    O.moe_unpermute(y, w, s2d, idx.shape[0], TOPK)
    t4 = time.perf_counter()
    total_rows = int(offsets[-1])
    ffn_est = ffn * total_rows / max(rows, 1)
    est = (t1 - t0) + (t2 - t1) + ffn_est + (t4 - t3)
    desc = (f"oracle port on the host: gating, permute and unpermute over all {idx.shape[0]} "
            f"tokens; expert FFN (fp32 GEMMs, as ref_grouped_gemm) timed on {rows} rows of "
            f"experts {experts} and scaled to all {total_rows} rows")
    return {"est_s": est, "desc": desc, "sample_experts": experts, "sample_rows": rows,
            "total_rows": total_rows, "gating_s": t1 - t0, "permute_s": t2 - t1,
            "ffn_sample_s": ffn, "ffn_scaled_s": ffn_est, "unpermute_s": t4 - t3}


def cpu_baseline_record(r, cores, value):
    return {"value": value, "unit": UNIT, "cores": cores, "cpu_model": cpu_model(),
            "kind": "port", "sample": r["desc"],
            "sample_experts": r["sample_experts"], "sample_rows": r["sample_rows"],
            "total_rows": r["total_rows"],
            "measured_s": {k: round(r[k], 6) for k in ("gating_s", "permute_s", "ffn_sample_s",
                                                      "unpermute_s")},
            "ffn_scaled_s": round(r["ffn_scaled_s"], 6)}


def _synthetic_module():
    """The seeded input generator, loaded by file path: it is pure torch, and
    loading it this way keeps the CPU arm free of the package __init__ (which
    needs the native extension), so `--impl reference` runs on a box where
    the CUDA build is missing."""
    import importlib.util
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "layerstormexpertkernels_b200",
                        "synthetic.py")
    spec = importlib.util.spec_from_file_location("_lsek_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cpu_inputs():
    token_inputs = _synthetic_module().token_inputs
    x = token_inputs(T_TOKENS, EXPERTS, HIDDEN, seed=0)
    return x.logits.numpy(), x.bias.numpy(), x.hidden.float().numpy()


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    logits, bias, hidden = cpu_inputs()
    per_step = []
    last = None
    for i in range(args.warmup + args.steps):
        last = cpu_layer_sample(logits, bias, hidden)
        if i >= args.warmup:
            per_step.append(last["est_s"])
    sec = statistics.mean(per_step)
    value = T_TOKENS / sec
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": T_TOKENS, "parallelism": "cpu"},
            "cpu_baseline": cpu_baseline_record(last, cores, value),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def host_pipeline_ms(forward, x, T, E, dev, steps, barrier, max_over_ranks):
    """The layer fed from pinned host memory through HostPipeline: every step
    copies its hidden rows and logits host->device and its output
    device->host, overlapped with the neighbouring steps' compute.  Device
    time from the first input copy to the last output copy, per step, max
    over ranks."""
    import torch
    import layerstormexpertkernels_b200 as P
    # Pinned buffers in this GPU's NUMA node (first touch under the GPU's
    # cores); the process's own affinity is restored afterwards.
    saved = os.sched_getaffinity(0)
    P.bind_host_to_device(dev)
    try:
        hidden_h, logits_h = x.hidden.pin_memory(), x.logits.pin_memory()
        outs_h = [torch.empty(T, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    finally:
        os.sched_setaffinity(0, saved)
    pipe = P.HostPipeline(forward, (T, HIDDEN), (T, E), dev)
    for i in range(2):
        pipe.submit(hidden_h, logits_h, outs_h[i % 2])
    pipe.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(pipe.h2d)
    for i in range(steps):
        pipe.submit(hidden_h, logits_h, outs_h[i % 2])
    e1.record(pipe.d2h)
    pipe.synchronize()
    barrier()
    return max_over_ranks(e0.elapsed_time(e1) / steps)


def gemm_roofline(kernel, flops, nbytes, ms, peaks, traffic=None):
    """Roofline of a GEMM launch against whichever floor is higher: its
    algorithmic bytes at the measured HBM copy bandwidth, or its FLOPs at the
    measured sustained bf16 rate (the GEMM runs inside a long step)."""
    gbs = nbytes / (ms * 1e-3) / 1e9
    tflops = flops / (ms * 1e-3) / 1e12
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
    t_tensor = flops / (peaks["bf16_tflops_sustained"] * 1e12)
    out = {"kernel": kernel, "algorithmic_bytes": nbytes, "flops": flops, "traffic": traffic,
           "hbm_gbs": gbs, "tensor_tflops": tflops,
           "tensor_frac_of_sustained": tflops / peaks["bf16_tflops_sustained"],
           "peak_source": peaks["source"]}
    if t_tensor > t_hbm:
        out.update({"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops_sustained"],
                    "unit": "TFLOP/s", "frac": tflops / peaks["bf16_tflops_sustained"]})
    else:
        out.update({"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": gbs / peaks["hbm_gbs"]})
    return out


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    T = args.tokens
    E = args.experts
    w_gu, w_down = expert_weights(E, HIDDEN, INTER, device=dev)
    x = token_inputs(T, E, HIDDEN, seed=rank)
    layer = P.MoELayer(w_gu, w_down, x.bias.to(dev), topk=TOPK, n_group=N_GROUP,
                       topk_group=TOPK_GROUP, routed_scaling_factor=RSF, renormalize=True,
                       max_tokens=T)
    hidden, logits = x.hidden.to(dev), x.logits.to(dev)
    out = torch.empty_like(hidden)
    tw = torch.empty(T, TOPK, dtype=torch.float32, device=dev)
    ti = torch.empty(T, TOPK, dtype=torch.int32, device=dev)

    for _ in range(args.warmup):
        layer(hidden, logits, out=out, topk_weights=tw, topk_indices=ti)
    torch.cuda.synchronize()
    if P.device_error() != 0:
        raise RuntimeError("a kernel reported a device-side error during warm-up")
    rows_per_expert = torch.bincount(ti.flatten().long(), minlength=E).cpu().numpy()

    # ---- timed region: K steps, stage events recorded on the launch stream
    stage_ev = [P.StageEvents() for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    start.record()
    for i in range(args.steps):
        layer(hidden, logits, out=out, stage_events=stage_ev[i])
    end.record()
    torch.cuda.synchronize()
    sampler.stop()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    per_step = [ev.elapsed_ms() for ev in stage_ev]
    stage_ms = {s: statistics.mean(d[s] for d in per_step) for s in STAGES}
    if P.device_error() != 0:
        raise RuntimeError("a kernel reported a device-side error in the timed region")

    # ---- end to end through the public call, host buffers, copies timed
    e2e_ms = host_pipeline_ms(lambda h, l: layer(h, l), x, T, E, dev, args.steps, barrier,
                              max_over_ranks)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    rows = T * TOPK
    touched = int((rows_per_expert > 0).sum())
    # Algorithmic bytes of the dominant kernel (gate/up GEMM + SwiGLU): the
    # weights of every touched expert once, the permuted rows once, the
    # activations written once.
    gu_bytes = touched * 2 * INTER * HIDDEN * 2 + rows * HIDDEN * 2 + rows * INTER * 2
    gu_flops = 2.0 * rows * HIDDEN * 2 * INTER
    dn_bytes = touched * HIDDEN * INTER * 2 + rows * INTER * 2 + rows * HIDDEN * 2
    dn_flops = 2.0 * rows * INTER * HIDDEN
    stage_bytes = {
        "gating": T * E * 4 + E * 4 + T * TOPK * 8,
        "route": T * TOPK * 4 * 3 + (E + 1) * 4,
        "row_copy": T * HIDDEN * 2 + rows * HIDDEN * 2,
        "gate_up_swiglu_gemm": gu_bytes,
        "down_gemm": dn_bytes,
        "unpermute": rows * HIDDEN * 2 + T * TOPK * 8 + T * HIDDEN * 2,
    }
    stages = {s: {"ms": stage_ms[s], "gbs": stage_bytes[s] / (stage_ms[s] * 1e-3) / 1e9,
                  "bytes": stage_bytes[s]} for s in STAGES}
    stages["gate_up_swiglu_gemm"]["tflops"] = gu_flops / (stage_ms["gate_up_swiglu_gemm"] * 1e-3) / 1e12
    stages["down_gemm"]["tflops"] = dn_flops / (stage_ms["down_gemm"] * 1e-3) / 1e12
    dom = "gate_up_swiglu_gemm"
    traffic = load_traffic().get(dom, {}).get("bytes_per_launch")
    roofline = gemm_roofline(dom, gu_flops, gu_bytes, stage_ms[dom], peaks, traffic)

    line = {"metric": METRIC, "value": world * T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded randn tokens; per-expert seeded N(0,0.02) bf16 weights)",
            "config": {"workload": WORKLOAD if (T, E) == (T_TOKENS, EXPERTS) else
                       f"profiling case: T={T}, E={E} (cfg1 otherwise)",
                       "tokens_per_gpu": T, "global_tokens": world * T,
                       "hidden": HIDDEN, "inter": INTER, "experts": E, "topk": TOPK,
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "inputs larger than L2: 22.5 GB of expert weights per step"},
            # gating, route (one kernel), row copy (T > 64; smaller T gathers the rows in the
            # gate/up GEMM's loads), gate/up GEMM, down GEMM, unpermute
            "gpu_launches": (5 + (T > 64)) * args.steps,
            "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": T * HIDDEN * 2 + T * E * 4,
                    "d2h_bytes_per_step": T * HIDDEN * 2,
                    "copies": "pinned host buffers, overlapped with compute (HostPipeline)"},
            "roofline": roofline,
            "stages": stages,
            "clocks": sampler.summary()}
    if world == 1 and (T, E) == (T_TOKENS, EXPERTS) and not args.no_sweeps:
        line["swiglu_sweep"] = swiglu_sweep(peaks)
        line["decode"] = decode_latency(layer, E, dev, peaks)
        line["gemm_compute_sweep"] = gemm_compute_sweep(w_gu, w_down, x.bias.to(dev), E, dev, peaks)
    if world == 1 and not args.no_cpu_baseline and (T, E) == (T_TOKENS, EXPERTS):
        import torch as _t
        cores = len(os.sched_getaffinity(0))
        _t.set_num_threads(cores)
        logits_np, bias_np, hidden_np = cpu_inputs()
        r = cpu_layer_sample(logits_np, bias_np, hidden_np)
        line["cpu_baseline"] = cpu_baseline_record(r, cores, T_TOKENS / r["est_s"])
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# SwiGLU sweep and decode latency (N = 1)
# ---------------------------------------------------------------------------

def _l2_flusher(dev):
    """Writes 256 MiB (twice the 126 MB L2) so the next kernel starts cold."""
    import torch
    buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    return lambda: buf.fill_(1)


def swiglu_sweep(peaks, reps=20):
    """cfg2: fused_swiglu on [N, 2*2048] bf16 ~ N(0,1) -> [N, 2048], N in
    {256 ... 65536}; 12,288 bytes per row; L2 flushed before every timed call."""
    import torch
    import layerstormexpertkernels_b200 as P
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = _l2_flusher(dev)
    out = {}
    for n in (256, 1024, 4096, 16384, 65536):
        g = torch.Generator(device=dev).manual_seed(n)
        x = torch.randn(n, 2 * INTER, generator=g, device=dev).to(torch.bfloat16)
        P.fused_swiglu(x)
        torch.cuda.synchronize()
        # All reps enqueued before one synchronize: the host runs ahead, so no
        # launch gap of the host falls between an event and its kernel.
        marks = []
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            P.fused_swiglu(x)
            b.record()
            marks.append((a, b))
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in marks)
        gbs = n * 12288 / (ms * 1e-3) / 1e9
        out[str(n)] = {"us": ms * 1e3, "gbs": gbs, "frac_of_hbm": gbs / peaks["hbm_gbs"]}
    return {"workload": "cfg2: fused_swiglu [N, 4096] -> [N, 2048] bf16, L2 flushed per call",
            "by_rows": out}


def decode_latency(layer, E, dev, peaks, reps=30):
    """cfg4: the whole layer at T in {1, 8, 32, 64} with the cfg1 weights
    resident; floor = bytes of the touched experts' weights / HBM bandwidth."""
    import torch
    from layerstormexpertkernels_b200.synthetic import token_inputs
    out = {}
    for t in (1, 8, 32, 64):
        x = token_inputs(t, E, HIDDEN, seed=1000 + t)
        hidden, logits = x.hidden.to(dev), x.logits.to(dev)
        y = torch.empty_like(hidden)
        ti = torch.empty(t, TOPK, dtype=torch.int32, device=dev)
        tw = torch.empty(t, TOPK, dtype=torch.float32, device=dev)
        for _ in range(3):
            layer(hidden, logits, out=y, topk_weights=tw, topk_indices=ti)
        torch.cuda.synchronize()
        touched = int(torch.unique(ti).numel())
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            layer(hidden, logits, out=y)
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        floor_bytes = touched * 3 * INTER * HIDDEN * 2
        floor_us = floor_bytes / (peaks["hbm_gbs"] * 1e9) * 1e6
        out[str(t)] = {"us": ms * 1e3, "touched_experts": touched, "floor_us": floor_us,
                       "frac_of_floor": floor_us / (ms * 1e3)}
        # The same call replayed from a CUDA graph (how a decode loop runs it):
        # no host launch gaps between the layer's kernels.
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                layer(hidden, logits, out=y)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                layer(hidden, logits, out=y)
            gtimes = []
            for _ in range(reps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                graph.replay()
                b.record()
                torch.cuda.synchronize()
                gtimes.append(a.elapsed_time(b))
            del graph
            gus = statistics.median(gtimes) * 1e3
            out[str(t)].update({"us_graph": gus, "frac_of_floor_graph": floor_us / gus})
        except RuntimeError as exc:
            out[str(t)]["us_graph"] = None
            out[str(t)]["graph_error"] = str(exc).splitlines()[0][:200]
    return {"workload": "cfg4: decode-shaped layer, T in {1, 8, 32, 64}, cfg1 weights resident "
                        "(22.5 GB, larger than L2, so touched experts stream from HBM); "
                        "us = eager call, us_graph = the call replayed from a CUDA graph",
            "by_tokens": out}


def gemm_compute_sweep(w_gu, w_down, bias, E, dev, peaks, reps=5):
    """The expert GEMMs where they are compute-bound: T in {16384, 32768}
    tokens (512 and 1024 rows per expert on average) on the resident cfg1
    weights; TFLOP/s against the measured sustained bf16 peak (seconds-long
    GEMMs run under the power cap)."""
    import torch
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import token_inputs
    out = {}
    for t in (16384, 32768):
        x = token_inputs(t, E, HIDDEN, seed=2000 + t)
        w, idx = P.topk_gating(x.logits.to(dev), bias, TOPK, N_GROUP, TOPK_GROUP, RSF, True)
        permuted, offs, _, _ = P.moe_permute(x.hidden.to(dev), idx, E)
        del x
        rows = permuted.shape[0]
        res = {}
        for name, fn, flops in (
                ("gate_up_swiglu", lambda: P.grouped_gemm_swiglu_bf16(permuted, w_gu, offs),
                 2.0 * rows * HIDDEN * 2 * INTER),
                ("down", None, 2.0 * rows * INTER * HIDDEN)):
            if fn is None:
                h = P.grouped_gemm_swiglu_bf16(permuted, w_gu, offs)
                fn = lambda h=h: P.grouped_gemm_bf16(h, w_down, offs)
            fn()
            torch.cuda.synchronize()
            times = []
            for _ in range(reps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                torch.cuda.synchronize()
                times.append(a.elapsed_time(b))
            ms = statistics.median(times)
            tf = flops / (ms * 1e-3) / 1e12
            res[name] = {"ms": ms, "tflops": tf,
                         "frac_of_sustained": tf / peaks["bf16_tflops_sustained"],
                         "frac_of_burst": tf / peaks["bf16_tflops"]}
        del permuted
        torch.cuda.empty_cache()
        out[str(t)] = res
    return {"workload": "expert GEMMs at T in {16384, 32768} tokens (E=256, top-8, cfg1 weights): "
                        "compute-bound", "by_tokens": out}


# ---------------------------------------------------------------------------
# Expert-parallel arm (N > 1)
# ---------------------------------------------------------------------------

NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s
CFG3_TOKENS = 8192


class Marker:
    """mark(name) records a CUDA event on the current stream; ms() gives the
    time between consecutive marks."""

    def __init__(self):
        import torch
        self.torch = torch
        self.events = []

    def mark(self, name):
        ev = self.torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events.append((name, ev))

    def ms(self) -> dict:
        out = {}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


def mean_stages(markers) -> dict:
    per = [m.ms() for m in markers]
    return {name: statistics.mean(p.get(name, 0.0) for p in per) for name in per[0]}


def route_launches(keys: int) -> int:
    """Kernels of one route (moe_permute's counting sort): one CTA up to 4096
    keys, else count + scan + rank."""
    return 1 if keys <= 4096 else 3


def run_ep(args):
    import torch
    import torch.distributed as dist

    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200 import ep as EP
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce(v: float, op) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    MAX = dist.ReduceOp.MAX if world > 1 else None
    SUM = dist.ReduceOp.SUM if world > 1 else None
    T, E = args.tokens, args.experts
    El = E // world
    w_gu, w_down = expert_weights(E, HIDDEN, INTER, device=dev,
                                  experts=list(range(rank * El, (rank + 1) * El)))
    x = token_inputs(T, E, HIDDEN, seed=rank)
    bias = token_inputs(T, E, 8, seed=0).bias.to(dev)  # rank 0's bias, shared by all ranks
    peer = args.transport == "peer"
    domain = EP.PeerDomain(max(T, CFG3_TOKENS), HIDDEN, TOPK) if peer else None
    layer = EP.EPMoELayer(w_gu, w_down, bias, E, topk=TOPK, n_group=N_GROUP,
                          topk_group=TOPK_GROUP, routed_scaling_factor=RSF, renormalize=True,
                          domain=domain, combine=args.combine, push_chunks=args.push_chunks)
    hidden, logits = x.hidden.to(dev), x.logits.to(dev)

    for _ in range(args.warmup):
        layer(hidden, logits)
    torch.cuda.synchronize()
    if P.device_error() != 0:
        raise RuntimeError("a kernel reported a device-side error during warm-up")
    w_r, idx_r = layer.gate(logits)
    if peer:
        d = EP.peer_dispatch(domain, hidden, idx_r, w_r, E)
        recv_rows, valid = d.recv_rows.shape[0], d.valid_slots
        # finish the epoch so every rank's flags stay in step
        _, _, s2d0, _ = P._C.ep_expert_permute(d.recv_rows, d.recv_ids, El, valid)
        EP.peer_combine(d, torch.zeros(valid, HIDDEN, dtype=torch.bfloat16, device=dev), s2d0)
    else:
        d = EP.dispatch(hidden, idx_r, w_r, E)
        recv_rows, valid = d.recv_rows.shape[0], d.valid_slots
    del d

    markers = [Marker() for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    start.record()
    for i in range(args.steps):
        mk = markers[i]
        mk.mark("start")
        layer(hidden, logits, mark=mk.mark)
    end.record()
    torch.cuda.synchronize()
    sampler.stop()
    barrier()
    ms = reduce(start.elapsed_time(end) / args.steps, MAX)
    stage_ms = mean_stages(markers)
    if P.device_error() != 0:
        raise RuntimeError("a kernel reported a device-side error in the timed region")

    # ---- end to end: pinned host tokens in, layer output out, every step
    e2e_ms = host_pipeline_ms(lambda h, l: layer(h, l), x, T, E, dev, args.steps, barrier,
                              lambda v: reduce(v, MAX))

    ep_combine = ep_combine_bench(args, dev, E, world, rank, reduce, MAX, SUM, barrier, domain)
    # The other transport's cfg3 numbers on the same ranks, for comparison.
    ep_combine_other = None
    if world > 1:
        other = None if peer else EP.PeerDomain(CFG3_TOKENS, HIDDEN, TOPK)
        try:
            ep_combine_other = ep_combine_bench(args, dev, E, world, rank, reduce, MAX, SUM,
                                                barrier, other)
        finally:
            if other is not None:
                other.close()

    plan = 1 + route_launches(T * world) + 1
    permute = route_launches(recv_rows * TOPK) + 1
    if peer and layer.combine == "push":
        # gating, plan, counts read, dispatch push, wait, permute, gate/up, scan, combine
        # plan, push_chunks - 1 x (down GEMM, combine push), last down GEMM, then per token
        # chunk a push and a wait (and a reduce when the chunk holds tokens), send-side scan
        C = domain.combine_chunks
        ct = -(-T // C)  # every rank has T tokens: the call's chunks cover them
        reduces = min(C, -(-T // ct))
        launches = (1 + plan + 1 + 1 + 1 + permute + 1 + 1 + 1 + 2 * (layer.push_chunks - 1)
                    + 1 + 2 * C + reduces + 1)
    elif peer:  # ... as above up to the combine plan, down+combine, wait, scan, reduce
        launches = 1 + plan + 1 + 1 + 1 + permute + 1 + 1 + 1 + 1 + 1 + 1 + 1
    else:     # gating, plan, pack, permute, gate/up, down, scan, combine pack, scan, reduce
        launches = 1 + plan + 1 + permute + 2 + 2 + 1 + 1
    if rank == 0:
        peaks = load_peaks()
        gu_flops = 2.0 * valid * HIDDEN * 2 * INTER
        gu_bytes = El * 2 * INTER * HIDDEN * 2 + valid * HIDDEN * 2 + valid * INTER * 2
        gu_ms = stage_ms["gate_up_swiglu_gemm"]
        if not peer:
            transport = "NCCL all-to-all dispatch/combine"
        elif layer.combine == "fused":
            transport = ("peer memory: dispatch kernel stores rows into the owner GPUs, combine "
                         "fused into the down-GEMM epilogue (NVLink stores), epoch flags")
        else:
            transport = ("peer memory: dispatch kernel stores rows into the owner GPUs, a combine "
                         "kernel streams the weighted rows back over NVLink, epoch flags")
        roofline = gemm_roofline("gate_up_swiglu_gemm (rank 0)", gu_flops, gu_bytes, gu_ms, peaks)
        line = {"metric": METRIC, "value": world * T / (ms * 1e-3), "unit": UNIT,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16",
                "data": "synthetic (seeded randn tokens per rank; per-expert seeded N(0,0.02) bf16 weights)",
                "config": {"workload": (f"cfg1 layer expert-parallel over {world} GPU(s): "
                                        f"T={T} tokens per GPU, E={E} ({El} per GPU), H={HIDDEN}, "
                                        f"I={INTER}, top-{TOPK}"),
                           "transport": transport,
                           "tokens_per_gpu": T, "global_tokens": world * T, "experts": E,
                           "experts_per_gpu": El, "parallelism": f"ep{world}",
                           "l2": "inputs larger than L2: expert weights and token rows per step"},
                "gpu_launches": launches * args.steps,
                "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": UNIT,
                        "h2d_bytes_per_step": T * HIDDEN * 2 + T * E * 4,
                        "d2h_bytes_per_step": T * HIDDEN * 2,
                        "copies": "pinned host buffers, overlapped with compute (HostPipeline)"},
                "roofline": roofline,
                "stages_rank0_ms": stage_ms,
                "ep_combine": ep_combine,
                "ep_combine_other_transport": ep_combine_other,
                "clocks": sampler.summary()}
        print(json.dumps(line), flush=True)
    if domain is not None:
        domain.close()
    if world > 1:
        dist.destroy_process_group()


def ep_combine_bench(args, dev, E, world, rank, reduce, MAX, SUM, barrier, domain=None):
    """dispatch + weighted combine of T=8192 tokens per
    rank with synthetic bf16 expert outputs (no GEMM); per-rank time is the
    max over ranks."""
    import torch

    from layerstormexpertkernels_b200 import ep as EP
    from layerstormexpertkernels_b200.synthetic import token_inputs

    T = CFG3_TOKENS
    El = E // world
    x = token_inputs(T, E, HIDDEN, seed=100 + rank)
    bias = token_inputs(T, E, 8, seed=100).bias.to(dev)
    hidden, logits = x.hidden.to(dev), x.logits.to(dev)
    import layerstormexpertkernels_b200 as P
    w, idx = P.topk_gating(logits, bias, TOPK, N_GROUP, TOPK_GROUP, RSF, True)
    g = torch.Generator(device=dev).manual_seed(rank)
    y_all = None

    def step(mk=None):
        nonlocal y_all
        mark = mk.mark if mk else None
        if mk:
            mk.mark("start")
        if domain is not None:
            d = EP.peer_dispatch(domain, hidden, idx, w, E, mark=mark)
            _, _, s2d, _ = P._C.ep_expert_permute(d.recv_rows, d.recv_ids, El, d.valid_slots)
        else:
            d = EP.dispatch(hidden, idx, w, E, mark=mark)
            _, _, s2d = EP.expert_permute(d, El)
        if y_all is None or y_all.shape[0] < d.valid_slots:
            y_all = torch.randn(d.valid_slots, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        if mk:
            mk.mark("ep_expert_permute")
        if domain is not None:
            return EP.peer_combine(d, y_all[:d.valid_slots], s2d, mark=mark)
        return EP.combine(d, y_all[:d.valid_slots], s2d, mark=mark)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    steps = max(args.steps, 5)
    marks = [Marker() for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        step(marks[i])
    torch.cuda.synchronize()
    barrier()
    st = mean_stages(marks)
    if domain is not None:
        # The peer combine is pushed and reduced in token chunks: its waits
        # run inside the reduce stream, so "ep_combine_push" is the pushes and
        # "ep_combine_reduce" the reduce work left after the last push.
        disp_names = ("ep_plan", "ep_dispatch_push", "ep_dispatch_wait", "ep_expert_permute")
        comb_names = ("ep_combine_push", "ep_combine_reduce")
        disp_x = st["ep_dispatch_push"] + st["ep_dispatch_wait"]
        comb_x = st["ep_combine_push"]
    else:
        disp_names = ("ep_plan", "ep_dispatch_pack", "ep_dispatch_exchange", "ep_expert_permute")
        comb_names = ("ep_combine_pack", "ep_combine_exchange", "ep_combine_reduce")
        disp_x = st["ep_dispatch_exchange"]
        comb_x = st["ep_combine_exchange"]
    disp = sum(st[n] for n in disp_names)
    comb = sum(st[n] for n in comb_names)
    per_rank = El
    own = torch.where((idx >= 0) & (idx < E), idx // per_rank, -1)
    off_slots = int(((own != rank) & (own >= 0)).sum().item())
    off_rows = 0
    for gg in range(world):
        if gg != rank:
            off_rows += int((own == gg).any(dim=1).sum().item())
    comb_bytes = off_slots * HIDDEN * 2
    disp_bytes = off_rows * HIDDEN * 2
    disp, comb = reduce(disp, MAX), reduce(comb, MAX)
    comb_x, disp_x = reduce(comb_x, MAX), reduce(disp_x, MAX)
    comb_bytes_all = reduce(float(comb_bytes), SUM)
    disp_bytes_all = reduce(float(disp_bytes), SUM)
    gbs = comb_bytes_all / world / (comb * 1e-3) / 1e9 if comb > 0 else 0.0
    return {"workload": (f"cfg3: T={T} tokens per rank, E={E} over {world} rank(s), H={HIDDEN} "
                         "bf16, top-8 sigmoid routing (8 groups / 4 kept), synthetic bf16 expert "
                         "outputs, weighted per-slot combine with fp32 accumulation"),
            "transport": ("peer (token-chunked: %d chunks)" % domain.combine_chunks
                          if domain is not None else "nccl all_to_all_single"),
            "stages_ms": st,
            "steps": steps,
            "dispatch_ms": disp, "combine_ms": comb,
            "dispatch_exchange_ms": disp_x, "combine_exchange_ms": comb_x,
            "combine_offrank_bytes_per_gpu": comb_bytes_all / world,
            "dispatch_offrank_bytes_per_gpu": disp_bytes_all / world,
            "combine_gbs_per_gpu": gbs,
            "combine_exchange_gbs_per_gpu": (comb_bytes_all / world / (comb_x * 1e-3) / 1e9
                                             if comb_x > 0 else 0.0),
            "dispatch_gbs_per_gpu": (disp_bytes_all / world / (disp * 1e-3) / 1e9
                                     if disp > 0 else 0.0),
            "nvlink_peak_gbs": NVLINK_GBS,
            "nvlink_peak_source": "measured peer copy per direction per GPU on this pool",
            "combine_frac_of_nvlink": gbs / NVLINK_GBS}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=T_TOKENS)
    ap.add_argument("--experts", type=int, default=EXPERTS,
                    help="routed experts (default 256); smaller values make profiling cases")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweeps", action="store_true",
                    help="skip the cfg2 SwiGLU sweep and the cfg4 decode latencies")
    ap.add_argument("--ep", action="store_true",
                    help="run the expert-parallel arm even on one GPU (default for N > 1)")
    ap.add_argument("--transport", choices=["peer", "nccl"], default="peer",
                    help="expert-parallel exchange: peer-memory kernels (default) or NCCL all-to-all")
    ap.add_argument("--combine", choices=["auto", "fused", "push"], default="auto",
                    help="peer transport: combine fused into the down GEMM, or a separate push "
                         "kernel (auto: push)")
    ap.add_argument("--push-chunks", type=int, default=2,
                    help="push combine: expert groups whose rows stream while the next computes")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.ep or dist_env()[1] > 1:
        run_ep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
