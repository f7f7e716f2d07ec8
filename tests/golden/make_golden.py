"""Generates the golden fixtures of tests/golden/ by running the reference's
own CPU torch implementation (tests/test_reference.py of
kkontosis/LayerStoRmExpertKernels) on seeded inputs.

The reference cannot travel to the GPU box, so its outputs are committed
here as small .npz files; tests/test_oracle_golden.py checks the oracle
against them and the GPU tests check the CUDA path against the oracle.

    python tests/golden/make_golden.py --ref /path/to/reference

Each case draws its inputs from torch.Generator().manual_seed(seed) on the
CPU.  Inputs too large to commit are stored as (seed, shape) plus a checksum;
tests/golden/cases.py regenerates them identically.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "tests", "test_reference.py")
    spec = importlib.util.spec_from_file_location("lsek_reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gating_cases(ref, out_dir):
    for c in cases.GATING_CASES:
        logits, bias = cases.gating_inputs(c)
        w, idx = ref.ref_topk_gating(
            logits, bias, topk=c["topk"], n_group=c["n_group"], topk_group=c["topk_group"],
            routed_scaling_factor=c["rsf"], renormalize=c["renorm"], scoring_func=c["scoring"])
        payload = dict(weights=w.numpy(), indices=idx.numpy(),
                       logits_sum=np.float64(logits.double().sum().item()))
        if logits.numel() <= 64 * 1024:
            payload["logits"] = logits.numpy()
            if bias is not None:
                payload["bias"] = bias.numpy()
        np.savez_compressed(os.path.join(out_dir, f"gating_{c['name']}.npz"), **payload)


def adaptive_cases(ref, out_dir):
    # Known-answer inputs of the reference test (test_reference.py:468-499).
    kw = torch.tensor([[0.50, 0.30, 0.15, 0.05], [0.90, 0.05, 0.03, 0.02],
                       [0.25, 0.25, 0.25, 0.25], [0.40, 0.35, 0.20, 0.05]], dtype=torch.float32)
    ki = torch.tensor([[10, 20, 30, 40], [5, 15, 25, 35], [1, 2, 3, 4], [100, 200, 300, 400]],
                      dtype=torch.int32)
    for name, (w, i, thr) in {
        "known_answer": (kw, ki, 0.9),
        "rand64": cases.adaptive_inputs(64, 8, seed=11) + (0.9,),
        "rand256_t05": cases.adaptive_inputs(256, 8, seed=12) + (0.5,),
        "rand32_k4_t1": cases.adaptive_inputs(32, 4, seed=13) + (1.0,),
    }.items():
        ow, oi, cnt = ref.ref_adaptive_gating(w, i, thr)
        np.savez_compressed(os.path.join(out_dir, f"adaptive_{name}.npz"), in_weights=w.numpy(),
                            in_indices=i.numpy(), threshold=np.float64(thr), weights=ow.numpy(),
                            indices=oi.numpy(), counts=cnt.numpy())


def swiglu_cases(ref, out_dir):
    for name, (n, d, scale, limit, seed) in {
        "plain": (64, 256, 1.0, 0.0, 21),
        "clamp10": (64, 256, 15.0, 10.0, 22),
        "edges": (4, 64, 40.0, 10.0, 23),
    }.items():
        g = torch.Generator().manual_seed(seed)
        gate = (torch.randn(n, d, generator=g) * scale).to(torch.bfloat16).float()
        up = (torch.randn(n, d, generator=g) * scale).to(torch.bfloat16).float()
        out = ref.ref_swiglu(gate, up, swiglu_limit=limit)
        np.savez_compressed(os.path.join(out_dir, f"swiglu_{name}.npz"), gate=gate.numpy(),
                            up=up.numpy(), limit=np.float64(limit), out=out.numpy())


def permute_cases(out_dir):
    # The reference's permute semantics (test_reference.py:534-558):
    # sort_idx = argsort(flat, stable=True); unsort_idx = argsort(sort_idx).
    for name, (T, k, E, sentinel_frac, seed) in {
        "t128_k4_e32": (128, 4, 32, 0.0, 31),
        "t96_k8_e64_sentinels": (96, 8, 64, 0.1, 32),
        "t1_k8_e256": (1, 8, 256, 0.0, 33),
        "t4096_k8_e256": (4096, 8, 256, 0.0, 34),
    }.items():
        idx = cases.permute_indices(T, k, E, sentinel_frac, seed)
        flat = idx.reshape(-1).long()
        key = torch.where(flat < 0, torch.full_like(flat, E), flat)
        sort_idx = torch.argsort(key, stable=True)
        unsort_idx = torch.argsort(sort_idx)
        counts = torch.bincount(key[key < E], minlength=E)
        offsets = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(counts, 0)])
        np.savez_compressed(os.path.join(out_dir, f"permute_{name}.npz"),
                            topk_indices=idx.numpy(), num_experts=np.int64(E),
                            perm=sort_idx.int().numpy(), s2d=unsort_idx.int().numpy(),
                            offsets=offsets.int().numpy())


def combine_cases(out_dir):
    # Per-slot and fixed-order reduce contracts of tests/test_kernels.py:113-129
    # and :168-185, evaluated with torch on the CPU.
    T, k, D, rows, seed = 24, 8, 256, 24 * 8, 41
    g = torch.Generator().manual_seed(seed)
    permuted = torch.randn(rows, D, generator=g).to(torch.bfloat16)
    weights = torch.rand(T, k, generator=g)
    s2d = torch.randperm(rows, generator=g).int()
    s = s2d.view(T, k)
    f32 = torch.zeros(T, k, D)
    b16 = torch.zeros(T, k, D, dtype=torch.bfloat16)
    for j in range(k):
        prod = weights[:, j:j + 1] * permuted[s[:, j].long()].float()
        f32[:, j, :] = prod
        b16[:, j, :] = prod.to(torch.bfloat16)
    red32 = torch.zeros(T, D)
    red16 = torch.zeros(T, D)
    for j in range(k):
        red32 += f32[:, j, :]
        red16 += b16[:, j, :].float()
    np.savez_compressed(os.path.join(out_dir, "combine_t24_k8_d256.npz"),
                        permuted=permuted.view(torch.int16).numpy().view(np.uint16),
                        weights=weights.numpy(), s2d=s2d.numpy(), perslot_f32=f32.numpy(),
                        perslot_bf16=b16.view(torch.int16).numpy().view(np.uint16),
                        reduce_f32=red32.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16),
                        reduce_bf16=red16.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def gemm_cases(ref, out_dir):
    g = torch.Generator().manual_seed(51)
    E, K, N = 4, 128, 64
    tokens = [8, 0, 16, 4]  # expert 1 empty, as in test_reference.py:501-532
    offsets = torch.tensor([0] + list(np.cumsum(tokens)), dtype=torch.int64)
    a = torch.randn(sum(tokens), K, generator=g).to(torch.bfloat16).float()
    w = [torch.randn(N, K, generator=g).to(torch.bfloat16).float() for _ in range(E)]
    out = ref.ref_grouped_gemm(a, w, offsets)
    np.savez_compressed(os.path.join(out_dir, "grouped_gemm_e4.npz"), a=a.numpy(),
                        b=torch.stack(w).numpy(), offsets=offsets.int().numpy(), out=out.numpy())

    # Expert FFN, top-1 routing (ref_expert_forward, test_reference.py:257-276).
    g = torch.Generator().manual_seed(52)
    B, H, I, E = 32, 256, 64, 4
    x = torch.randn(B, H, generator=g).to(torch.bfloat16).float()
    ids = torch.randint(0, E, (B,), generator=g)
    wg = [(torch.randn(I, H, generator=g) * 0.05).to(torch.bfloat16).float() for _ in range(E)]
    wu = [(torch.randn(I, H, generator=g) * 0.05).to(torch.bfloat16).float() for _ in range(E)]
    wd = [(torch.randn(H, I, generator=g) * 0.05).to(torch.bfloat16).float() for _ in range(E)]
    scores = torch.rand(B, generator=g)
    out = ref.ref_expert_forward(x, ids, wg, wu, wd, scores, E)
    np.savez_compressed(os.path.join(out_dir, "expert_forward_top1.npz"), x=x.numpy(),
                        ids=ids.int().numpy(), w_gate=torch.stack(wg).numpy(),
                        w_up=torch.stack(wu).numpy(), w_down=torch.stack(wd).numpy(),
                        scores=scores.numpy(), out=out.numpy())


def quant_cases(ref, out_dir):
    """FP8 E4M3 block quantisation / dequantisation and NVFP4 dequantisation
    (test_reference.py:19-107)."""
    g = torch.Generator().manual_seed(61)
    M, K = 6, 300  # 300 = two full 128-blocks and a ragged 44-wide one
    x = torch.randn(M, K, generator=g)
    x[1] *= 1000.0                 # large magnitudes
    x[2, 128:256] = 0.0            # an all-zero block: scale 1.0
    x[3] *= 1e-6                   # tiny magnitudes
    x[4] = x[4].to(torch.bfloat16).float()  # bf16 inputs, as the layer's activations
    x[5, :8] = torch.tensor([448.0, -448.0, 1.0, -1.0, 0.5, 3.0, -7.0, 0.0])
    q, scales = ref.ref_dynamic_fp8_quant(x)
    deq = ref.ref_fp8_dequant(q, scales, M, K)
    np.savez_compressed(os.path.join(out_dir, "fp8_quant_m6_k300.npz"), x=x.numpy(),
                        q=q.numpy(), scales=scales.numpy(), deq=deq.numpy())

    M, N = 4, 64
    packed = torch.randint(0, 256, (M, N // 2), generator=g, dtype=torch.int64).to(torch.uint8)
    scales = torch.pow(2.0, torch.randint(-4, 5, (M, N // 16), generator=g).float())
    out = ref.ref_nvfp4_dequant(packed, scales, M, N)
    np.savez_compressed(os.path.join(out_dir, "nvfp4_dequant_m4_n64.npz"), packed=packed.numpy(),
                        scales=scales.numpy(), out=out.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LSEK_REFERENCE"),
                    help="checkout of the reference project (or set LSEK_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", choices=["quant"], default=None,
                    help="write only this group of fixtures")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set LSEK_REFERENCE to the reference checkout")
    ref = load_reference(args.ref)
    if args.only == "quant":
        quant_cases(ref, args.out)
        print("wrote fixtures to", args.out)
        return
    gating_cases(ref, args.out)
    adaptive_cases(ref, args.out)
    swiglu_cases(ref, args.out)
    permute_cases(args.out)
    combine_cases(args.out)
    gemm_cases(ref, args.out)
    quant_cases(ref, args.out)
    print("wrote fixtures to", args.out)


if __name__ == "__main__":
    main()
