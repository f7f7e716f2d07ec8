"""One rank of the 2-GPU EP parity test (launched by torch.distributed.run
from tests/test_gpu_ep.py): runs the EP layer three times over the chosen
transport ("nccl": all-to-alls; "peer": peer-memory kernels with the combine
fused into the down GEMM; "peer-push": peer memory with a separate combine
kernel; "replicated": every rank holds the same tokens and the per-slot
rows are SUM all-reduced), then the
one-GPU canonical path on this rank's tokens with all experts, and writes
"bit-exact" to <out_dir>/ok<rank> when every call agrees.  With a third
argument "cfg3" the shapes are BASELINE cfg3's: 8192 tokens per rank, 256
experts, H = 7168, I = 2048, top-8."""
from __future__ import annotations

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def main(out_dir: str, transport: str, shape: str = "small") -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    try:
        import layerstormexpertkernels_b200 as P
        from test_gpu_ep import E_L, H_L, K_L, _layer_setup, canonical_gpu
        from layerstormexpertkernels_b200.ep import EPMoELayer, PeerDomain

        if shape == "cfg3":
            from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs
            E_L, H_L, K_L = 256, 7168, 8
            tokens = [8192] * world
            w_gu, w_down = expert_weights(E_L, H_L, 2048, device="cuda", seed_base=9000)
            toks = [token_inputs(t, E_L, H_L, seed=300 + r) for r, t in enumerate(tokens)]
        else:
            tokens = [300 + 57 * r for r in range(world)]
            w_gu, w_down, toks = _layer_setup(world, tokens)
        El = E_L // world
        bias = toks[0].bias.cuda()
        dom = PeerDomain(max(tokens), H_L, K_L) if transport.startswith("peer") else None
        combine = "push" if transport == "peer-push" else "fused"
        layer = EPMoELayer(w_gu[rank * El:(rank + 1) * El].contiguous(),
                           w_down[rank * El:(rank + 1) * El].contiguous(), bias, E_L, topk=K_L,
                           domain=dom, combine=combine)
        if transport == "replicated":  # every rank holds rank 0's tokens
            from layerstormexpertkernels_b200.ep import replicated_forward
            ref = canonical_gpu(toks[0], w_gu, w_down, bias, E_L, K_L)
            run = lambda: replicated_forward(
                toks[0].hidden.cuda(), toks[0].logits.cuda(), bias,
                w_gu[rank * El:(rank + 1) * El].contiguous(),
                w_down[rank * El:(rank + 1) * El].contiguous(), E_L, topk=K_L)
        else:
            ref = canonical_gpu(toks[rank], w_gu, w_down, bias, E_L, K_L)
            run = lambda: layer(toks[rank].hidden.cuda(), toks[rank].logits.cuda())
        same = True
        for _ in range(3):
            out = run()
            same &= torch.equal(out.view(torch.int16), ref.view(torch.int16))
        torch.cuda.synchronize()
        same &= P.device_error() == 0
        if dom is not None:
            dom.close()
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("bit-exact" if same else "differs")
        dist.barrier()
        return 0 if same else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "nccl",
                  sys.argv[3] if len(sys.argv) > 3 else "small"))
