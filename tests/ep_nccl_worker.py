"""One rank of the 2-GPU EP parity test (launched by torch.distributed.run
from tests/test_gpu_ep.py): runs the EP layer over NCCL, then the one-GPU
canonical path on this rank's tokens with all experts, and writes
"bit-exact" to <out_dir>/ok<rank> when the two agree."""
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


def main(out_dir: str) -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    try:
        from test_gpu_ep import E_L, K_L, _layer_setup, canonical_gpu
        from layerstormexpertkernels_b200.ep import EPMoELayer

        tokens = [300 + 57 * r for r in range(world)]
        w_gu, w_down, toks = _layer_setup(world, tokens)
        El = E_L // world
        bias = toks[0].bias.cuda()
        layer = EPMoELayer(w_gu[rank * El:(rank + 1) * El].contiguous(),
                           w_down[rank * El:(rank + 1) * El].contiguous(), bias, E_L, topk=K_L)
        out = layer(toks[rank].hidden.cuda(), toks[rank].logits.cuda())
        ref = canonical_gpu(toks[rank], w_gu, w_down, bias)
        same = torch.equal(out.view(torch.int16), ref.view(torch.int16))
        torch.cuda.synchronize()
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("bit-exact" if same else "differs")
        dist.barrier()
        return 0 if same else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main(sys.argv[1]))
