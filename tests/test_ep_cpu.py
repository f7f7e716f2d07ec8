"""Expert-parallel dispatch/combine on the CPU.

1. The restated EP steps (oracle/ep_oracle.py), composed over G simulated
   ranks, equal the reference's canonical one-rank per-slot combine bit for
   bit (moe_unpermute_bf16_perslot + moe_combine_reduce_slots_bf16_to_bf16,
   smxx/permute/moe_permute.h:67-99; tests/test_kernels.py:131-142, 187-200).
2. The EP host logic of layerstormexpertkernels_b200.ep (counts exchange,
   split sizes, exchange order, combine) run as 2 gloo ranks with the CPU
   steps equals the one-rank canonical layer on the union of the ranks'
   tokens."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep_oracle as EO
from oracle import moe_oracle as MO


def _routing(T, E, topk, seed, invalid=False):
    rng = np.random.default_rng(seed)
    idx = np.array([rng.choice(E, topk, replace=False) for _ in range(T)],
                   dtype=np.int32).reshape(T, topk)
    if invalid and T:
        idx[0, -1] = -1
        idx[T // 2, 0] = E + 3
    w = rng.random((T, topk), dtype=np.float32)
    hidden = MO.bf16_round(rng.standard_normal((T, 64), dtype=np.float32))
    return hidden, idx, w


def _expert_fn(E, G):
    El = E // G

    def fn(rank, permuted, off):
        y = np.zeros_like(permuted, dtype=np.float32)
        for el in range(El):
            s, t = int(off[el]), int(off[el + 1])
            e = rank * El + el
            y[s:t] = MO.bf16_round((permuted[s:t] * np.float32(1.0 + 0.03 * e) + np.float32(0.01 * e))
                                   .astype(np.float32))
        return y
    return fn


def _canonical(hidden, idx, w, E, fn):
    """One rank, all experts: permute -> fn -> per-slot bf16 -> fixed-order reduce."""
    permuted, off, s2d, _ = MO.moe_permute(hidden, idx, E)
    y = np.zeros((permuted.shape[0], hidden.shape[1]), dtype=np.float32)
    valid = int(off[E])
    y[:valid] = fn(0, permuted[:valid], off)
    return MO.reduce_slots(MO.moe_unpermute_perslot_bf16(y, w, s2d, idx.shape[0], idx.shape[1]))


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("T", [0, 1, 37])
def test_ep_composition_equals_canonical_combine(G, T):
    E, topk = 32, 4
    ranks = [_routing(T + r, E, topk, seed=10 * G + r, invalid=(r == 0)) for r in range(G)]
    outs = EO.ep_reference([r[0] for r in ranks], [r[1] for r in ranks], [r[2] for r in ranks], E,
                           _expert_fn(E, G))
    one = _expert_fn(E, 1)
    for r in range(G):
        hidden, idx, w = ranks[r]
        ref = _canonical(hidden, idx, w, E, one)
        assert outs[r].shape == ref.shape
        assert np.array_equal(outs[r].view(np.uint32), ref.view(np.uint32))


def test_plan_orders_rows_rank_major_by_token():
    E, G = 16, 4
    idx = np.array([[0, 5], [12, 13], [4, 1], [9, 15]], dtype=np.int32)  # owners: {0,1},{3},{1,0},{2,3}
    off, counts, pair_row, row_pair = EO.ep_plan(idx, E, G)
    assert off.tolist() == [0, 2, 4, 5, 7]
    assert counts.tolist() == [[2, 2], [2, 2], [1, 1], [2, 3]]
    pr = pair_row.reshape(4, G)
    # rank 0 rows: tokens 0, 2; rank 1: tokens 0, 2; rank 2: token 3; rank 3: tokens 1, 3
    assert [pr[0, 0], pr[2, 0], pr[0, 1], pr[2, 1], pr[3, 2], pr[1, 3], pr[3, 3]] == list(range(7))
    assert all(pr[t, g] >= 7 for t, g in [(1, 0), (3, 0), (1, 1), (3, 1), (0, 2), (1, 2), (2, 2),
                                           (0, 3), (2, 3)])
    assert np.array_equal(np.sort(row_pair), np.arange(16))


# ---------------------------------------------------------------------------
# gloo, world size 2: the host logic of ep.py
# ---------------------------------------------------------------------------

E_G, H_G, I_G, K_G = 16, 64, 32, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_inputs():
    rng = np.random.default_rng(7)
    w_gu = MO.bf16_round(rng.standard_normal((E_G, 2 * I_G, H_G), dtype=np.float32) * 0.1)
    w_down = MO.bf16_round(rng.standard_normal((E_G, H_G, I_G), dtype=np.float32) * 0.1)
    bias = (rng.standard_normal(E_G, dtype=np.float32) * 0.01).astype(np.float32)
    toks = []
    for r in range(2):
        T = 9 + 4 * r
        logits = rng.standard_normal((T, E_G), dtype=np.float32)
        hidden = MO.bf16_round(rng.standard_normal((T, H_G), dtype=np.float32))
        toks.append((hidden, logits))
    return w_gu, w_down, bias, toks


def _gloo_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ep_cpu_steps import CpuSteps
        from layerstormexpertkernels_b200.ep import EPMoELayer

        w_gu, w_down, bias, toks = _layer_inputs()
        El = E_G // world
        sl = slice(rank * El, (rank + 1) * El)
        layer = EPMoELayer(torch.from_numpy(w_gu[sl]).to(torch.bfloat16),
                           torch.from_numpy(w_down[sl]).to(torch.bfloat16), torch.from_numpy(bias),
                           E_G, topk=K_G, n_group=4, topk_group=2, steps=CpuSteps)
        hidden, logits = toks[rank]
        marks = []
        out = layer(torch.from_numpy(hidden).to(torch.bfloat16), torch.from_numpy(logits),
                    mark=marks.append)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.float().numpy())
        np.save(os.path.join(out_dir, f"marks{rank}.npy"), np.array(marks))
    finally:
        dist.destroy_process_group()


def test_ep_layer_gloo_world2_matches_one_rank(tmp_path):
    mp.spawn(_gloo_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    from ep_cpu_steps import canonical_layer
    w_gu, w_down, bias, toks = _layer_inputs()
    for r in range(2):
        hidden, logits = toks[r]
        ref = canonical_layer(hidden, logits, bias, w_gu, w_down, topk=K_G, n_group=4,
                              topk_group=2)
        got = np.load(tmp_path / f"out{r}.npy")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        marks = list(np.load(tmp_path / f"marks{r}.npy"))
        assert marks[0] == "gating" and marks[-1] == "ep_combine_reduce"


def test_ep_layer_one_rank_without_process_group():
    from ep_cpu_steps import CpuSteps, canonical_layer
    from layerstormexpertkernels_b200.ep import EPMoELayer
    w_gu, w_down, bias, toks = _layer_inputs()
    layer = EPMoELayer(torch.from_numpy(w_gu).to(torch.bfloat16),
                       torch.from_numpy(w_down).to(torch.bfloat16), torch.from_numpy(bias), E_G,
                       topk=K_G, n_group=4, topk_group=2, steps=CpuSteps)
    hidden, logits = toks[1]
    out = layer(torch.from_numpy(hidden).to(torch.bfloat16), torch.from_numpy(logits))
    ref = canonical_layer(hidden, logits, bias, w_gu, w_down, topk=K_G, n_group=4, topk_group=2)
    assert np.array_equal(out.float().numpy().view(np.uint32), ref.view(np.uint32))


def test_ep_layer_rejects_bad_sharding():
    from layerstormexpertkernels_b200.ep import EPMoELayer
    w = torch.zeros(3, 8, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        EPMoELayer(w, w, None, 16)


@pytest.mark.parametrize("G", [1, 4, 8])
def test_ep_layer_loopback_threads(G):
    """The same host logic with G ranks as threads (in-process exchange)."""
    from ep_cpu_steps import CpuSteps, canonical_layer
    from ep_loopback import LoopbackHub
    from layerstormexpertkernels_b200.ep import EPMoELayer

    w_gu, w_down, bias, _ = _layer_inputs()
    rng = np.random.default_rng(G)
    toks = [(MO.bf16_round(rng.standard_normal((5 + r, H_G), dtype=np.float32)),
             rng.standard_normal((5 + r, E_G), dtype=np.float32)) for r in range(G)]
    El = E_G // G

    def rank_fn(r, ex):
        sl = slice(r * El, (r + 1) * El)
        layer = EPMoELayer(torch.from_numpy(w_gu[sl]).to(torch.bfloat16),
                           torch.from_numpy(w_down[sl]).to(torch.bfloat16),
                           torch.from_numpy(bias), E_G, topk=K_G, n_group=4, topk_group=2,
                           group=ex, steps=CpuSteps)
        hidden, logits = toks[r]
        return layer(torch.from_numpy(hidden).to(torch.bfloat16), torch.from_numpy(logits))

    outs = LoopbackHub(G).run(rank_fn)
    for r in range(G):
        hidden, logits = toks[r]
        ref = canonical_layer(hidden, logits, bias, w_gu, w_down, topk=K_G, n_group=4,
                              topk_group=2)
        assert np.array_equal(outs[r].float().numpy().view(np.uint32), ref.view(np.uint32))


def _replicated_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ep_cpu_steps import CpuSteps
        from layerstormexpertkernels_b200.ep import replicated_forward

        w_gu, w_down, bias, toks = _layer_inputs()
        El = E_G // world
        sl = slice(rank * El, (rank + 1) * El)
        hidden, logits = toks[0]  # every rank holds the same tokens
        out = replicated_forward(torch.from_numpy(hidden).to(torch.bfloat16),
                                 torch.from_numpy(logits), torch.from_numpy(bias),
                                 torch.from_numpy(w_gu[sl]).to(torch.bfloat16),
                                 torch.from_numpy(w_down[sl]).to(torch.bfloat16), E_G, topk=K_G,
                                 n_group=4, topk_group=2, steps=CpuSteps)
        np.save(os.path.join(out_dir, f"rep{rank}.npy"), out.float().numpy())
    finally:
        dist.destroy_process_group()


def test_replicated_mode_gloo_world2(tmp_path):
    """The reference consumer's contract (replicated tokens, bf16 SUM
    all-reduce of the per-slot rows) gives the one-rank bits on every rank."""
    mp.spawn(_replicated_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    from ep_cpu_steps import canonical_layer
    w_gu, w_down, bias, toks = _layer_inputs()
    hidden, logits = toks[0]
    ref = canonical_layer(hidden, logits, bias, w_gu, w_down, topk=K_G, n_group=4, topk_group=2)
    for r in range(2):
        got = np.load(tmp_path / f"rep{r}.npy")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("G", [1, 4])
def test_replicated_mode_loopback_threads(G):
    from ep_cpu_steps import CpuSteps, canonical_layer
    from ep_loopback import LoopbackHub
    from layerstormexpertkernels_b200.ep import replicated_forward

    w_gu, w_down, bias, toks = _layer_inputs()
    hidden, logits = toks[1]
    El = E_G // G

    def rank_fn(r, ex):
        sl = slice(r * El, (r + 1) * El)
        return replicated_forward(torch.from_numpy(hidden).to(torch.bfloat16),
                                  torch.from_numpy(logits), torch.from_numpy(bias),
                                  torch.from_numpy(w_gu[sl]).to(torch.bfloat16),
                                  torch.from_numpy(w_down[sl]).to(torch.bfloat16), E_G, topk=K_G,
                                  n_group=4, topk_group=2, group=ex, steps=CpuSteps)

    outs = LoopbackHub(G).run(rank_fn)
    ref = canonical_layer(hidden, logits, bias, w_gu, w_down, topk=K_G, n_group=4, topk_group=2)
    for r in range(G):
        assert np.array_equal(outs[r].float().numpy().view(np.uint32), ref.view(np.uint32))


def _lost_rank_worker(rank, world, port, out_dir):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:  # this rank leaves between layer calls, with nothing in flight
        dist.destroy_process_group()
        return
    from ep_cpu_steps import CpuSteps
    from layerstormexpertkernels_b200.ep import EPMoELayer
    w_gu, w_down, bias, toks = _layer_inputs()
    El = E_G // world
    layer = EPMoELayer(torch.from_numpy(w_gu[:El]).to(torch.bfloat16),
                       torch.from_numpy(w_down[:El]).to(torch.bfloat16), torch.from_numpy(bias),
                       E_G, topk=K_G, n_group=4, topk_group=2, steps=CpuSteps)
    hidden, logits = toks[0]
    import time
    t0 = time.time()
    try:
        layer(torch.from_numpy(hidden).to(torch.bfloat16), torch.from_numpy(logits))
        outcome = "returned"
    except RuntimeError as exc:
        outcome = "error: " + type(exc).__name__
    with open(os.path.join(out_dir, "lost.txt"), "w") as f:
        f.write(f"{outcome} {time.time() - t0:.1f}")
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - the group is already broken
        pass


def test_ep_layer_lost_rank_raises_instead_of_hanging(tmp_path):
    """A rank that leaves the group makes the next EP layer call on the
    others fail with an error within the process-group timeout (5 s here),
    not hang: the counts exchange is the first collective of the layer."""
    mp.spawn(_lost_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    outcome, seconds = (tmp_path / "lost.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("error"), outcome
    assert float(seconds) < 60
