"""GPU parity of the expert-parallel dispatch/combine kernels.

1. Each EP kernel against its CPU restatement (oracle/ep_oracle.py), bit
   for bit, for world sizes 1-8 and sizes on both sides of the one-CTA route.
2. The whole EP layer (layerstormexpertkernels_b200.ep) with G ranks run as
   threads on one GPU, against the one-GPU canonical path made of the
   reference-surface ops (topk_gating, moe_permute, the grouped GEMMs,
   moe_unpermute_bf16_perslot, moe_combine_reduce_slots_bf16_to_bf16):
   identical bits for every G.
3. The peer-memory path (dispatch pushed into the owner ranks, combine
   fused into the down-GEMM epilogue) with one rank, its bounded waits, and
   both transports with 2 processes when the box has 2 GPUs."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from gpu_util import bits, bf16_dev, dev, f32, sync_and_check_device_error
from oracle import ep_oracle as EO
from oracle import moe_oracle as MO

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _routing(T, E, k, seed, invalid=True):
    rng = np.random.default_rng(seed)
    idx = np.array([rng.choice(E, k, replace=False) for _ in range(T)],
                   dtype=np.int32).reshape(T, k)
    if invalid and T > 2:
        idx[1, 0] = -1
        idx[T - 1, k - 1] = E + 5
    w = rng.random((T, k), dtype=np.float32)
    return idx, w


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("T", [0, 1, 37, 700, 5000])
def test_plan_matches_oracle(G, T):
    import layerstormexpertkernels_b200 as P
    E, k = 64, 8
    idx, _ = _routing(T, E, k, seed=T * 10 + G)
    off, counts, pair_row, row_pair = P._C.ep_plan(dev(idx), E, G)
    sync_and_check_device_error()
    o_off, o_counts, o_pr, o_rp = EO.ep_plan(idx, E, G)
    assert off.cpu().numpy().tolist() == o_off.tolist()
    assert counts.cpu().numpy().tolist() == o_counts.tolist()
    if T:
        assert np.array_equal(pair_row.cpu().numpy(), o_pr)
        assert np.array_equal(row_pair.cpu().numpy(), o_rp)


@pytest.mark.parametrize("G", [1, 2, 8])
@pytest.mark.parametrize("T,H", [(1, 64), (37, 7168), (700, 256)])
def test_dispatch_pack_and_slot_scan(G, T, H):
    import layerstormexpertkernels_b200 as P
    E, k = 64, 8
    idx, w = _routing(T, E, k, seed=T + G)
    hidden = MO.bf16_round(np.random.default_rng(T).standard_normal((T, H), dtype=np.float32))
    off, counts, pair_row, _ = P._C.ep_plan(dev(idx), E, G)
    rows = int(off[G].item())
    sr, sid, sw = P._C.ep_dispatch_pack(bf16_dev(hidden), dev(idx), dev(w), pair_row, off, rows,
                                        E, G)
    scan = P._C.ep_slot_scan(sid)
    sync_and_check_device_error()
    o_sr, o_sid, o_sw = EO.ep_dispatch_pack(hidden, idx, w, pair_row.cpu().numpy(),
                                            off.cpu().numpy(), E, G)
    assert np.array_equal(bits(sr), MO.bf16_bits(o_sr))
    assert np.array_equal(sid.cpu().numpy(), o_sid)
    assert np.array_equal(sw.cpu().numpy().view(np.uint32), o_sw.view(np.uint32))
    assert np.array_equal(scan.cpu().numpy(), EO.ep_slot_scan(o_sid))
    assert int(scan[-1].item()) == int(counts[:, 1].sum().item())


@pytest.mark.parametrize("R,El,k,H", [(1, 4, 8, 64), (300, 32, 8, 256), (1500, 32, 8, 128),
                                      (200, 1, 4, 7168)])
def test_expert_permute_and_combine(R, El, k, H):
    """Expert side: permute with -1 sentinels (multi-CTA route above 4096
    slots), then the weighted per-slot pack; sender side: the reduce."""
    import layerstormexpertkernels_b200 as P
    rng = np.random.default_rng(R + El)
    ids = rng.integers(-1, El, size=(R, k)).astype(np.int32)
    w = np.where(ids >= 0, rng.random((R, k), dtype=np.float32), 0).astype(np.float32)
    rows = MO.bf16_round(rng.standard_normal((R, H), dtype=np.float32))
    nv = int((ids >= 0).sum())
    permuted, offs, s2d, perm = P._C.ep_expert_permute(bf16_dev(rows), dev(ids), El, nv)
    sync_and_check_device_error()
    o_p, o_off, o_s2d, o_perm = EO.ep_expert_permute(rows, ids, El)
    assert offs.cpu().numpy().tolist() == o_off.tolist()
    assert np.array_equal(s2d.cpu().numpy(), o_s2d)
    assert np.array_equal(perm.cpu().numpy(), o_perm)
    assert np.array_equal(bits(permuted), MO.bf16_bits(o_p))
    # a synthetic expert output per permuted row
    y = MO.bf16_round(rng.standard_normal((nv, H), dtype=np.float32))
    slot_row = P._C.ep_slot_scan(dev(ids))
    comb = P._C.ep_combine_pack(bf16_dev(y), s2d, dev(ids), dev(w), slot_row, nv)
    sync_and_check_device_error()
    o_comb = EO.ep_combine_pack(y, o_s2d, ids, w, slot_row.cpu().numpy())
    assert np.array_equal(bits(comb), MO.bf16_bits(o_comb))


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("T,H", [(1, 64), (100, 7168), (900, 256)])
def test_combine_reduce_matches_oracle(G, T, H):
    import layerstormexpertkernels_b200 as P
    E, k = 64, 8
    idx, _ = _routing(T, E, k, seed=7 * T + G)
    off, counts, pair_row, _ = EO.ep_plan(idx, E, G)
    send_ids = EO.ep_dispatch_pack(np.zeros((T, 8), np.float32), idx, np.ones((T, k), np.float32),
                                   pair_row, off, E, G)[1]
    slot_row = EO.ep_slot_scan(send_ids)
    comb = MO.bf16_round(np.random.default_rng(T).standard_normal((int(slot_row[-1]), H),
                                                                   dtype=np.float32))
    out = P._C.ep_combine_reduce(bf16_dev(comb), dev(idx), dev(pair_row), dev(slot_row), E, G)
    sync_and_check_device_error()
    ref = EO.ep_combine_reduce(comb, idx, pair_row, slot_row, E, G)
    assert np.array_equal(bits(out), MO.bf16_bits(ref))


# ---------------------------------------------------------------------------
# the whole EP layer: G ranks as threads on one GPU
# ---------------------------------------------------------------------------

E_L, H_L, I_L, K_L = 64, 512, 256, 8


def _layer_setup(G, tokens):
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs
    w_gu, w_down = expert_weights(E_L, H_L, I_L, device="cuda", seed_base=7000)
    toks = [token_inputs(tokens[r], E_L, H_L, seed=100 + r) for r in range(G)]
    return w_gu, w_down, toks


def canonical_gpu(x, w_gu, w_down, bias, E=E_L, k=K_L):
    """The one-GPU canonical path through the reference-surface ops."""
    import layerstormexpertkernels_b200 as P
    hidden, logits = x.hidden.cuda(), x.logits.cuda()
    w, idx = P.topk_gating(logits, bias, k, 8, 4, 2.5, True)
    permuted, offs, s2d, _ = P.moe_permute(hidden, idx, E)
    h = P.grouped_gemm_swiglu_bf16(permuted, w_gu, offs)
    y = P.grouped_gemm_bf16(h, w_down, offs)
    perslot = P.moe_unpermute_bf16_perslot(y, w, s2d, hidden.shape[0], k)
    return P.moe_combine_reduce_slots_bf16_to_bf16(perslot)


@pytest.mark.parametrize("G,tokens", [(1, [300]), (2, [300, 257]), (4, [64, 1, 200, 90]),
                                      (8, [130] * 8)])
def test_ep_layer_threads_bit_exact(G, tokens):
    from ep_loopback import LoopbackHub
    from layerstormexpertkernels_b200.ep import EPMoELayer

    w_gu, w_down, toks = _layer_setup(G, tokens)
    bias = toks[0].bias.cuda()
    El = E_L // G
    stages = [[] for _ in range(G)]

    def rank_fn(r, ex):
        layer = EPMoELayer(w_gu[r * El:(r + 1) * El].contiguous(),
                           w_down[r * El:(r + 1) * El].contiguous(), bias, E_L, topk=K_L,
                           group=ex)
        return layer(toks[r].hidden.cuda(), toks[r].logits.cuda(), mark=stages[r].append)

    outs = LoopbackHub(G).run(rank_fn)
    sync_and_check_device_error()
    for r in range(G):
        ref = canonical_gpu(toks[r], w_gu, w_down, bias)
        assert torch.equal(outs[r].view(torch.int16), ref.view(torch.int16)), f"rank {r}"
        assert stages[r][0] == "gating" and stages[r][-1] == "ep_combine_reduce"


@pytest.mark.parametrize("G", [2, 4])
def test_replicated_mode_threads_bit_exact(G):
    """The reference consumer's contract: replicated tokens, local experts'
    per-slot rows, SUM all-reduce (in-process here), fixed-order reduce."""
    from ep_loopback import LoopbackHub
    from layerstormexpertkernels_b200.ep import replicated_forward

    w_gu, w_down, toks = _layer_setup(1, [333])
    bias = toks[0].bias.cuda()
    El = E_L // G

    def rank_fn(r, ex):
        return replicated_forward(toks[0].hidden.cuda(), toks[0].logits.cuda(), bias,
                                  w_gu[r * El:(r + 1) * El].contiguous(),
                                  w_down[r * El:(r + 1) * El].contiguous(), E_L, topk=K_L,
                                  group=ex)

    outs = LoopbackHub(G).run(rank_fn)
    sync_and_check_device_error()
    ref = canonical_gpu(toks[0], w_gu, w_down, bias)
    for r in range(G):
        assert torch.equal(outs[r].view(torch.int16), ref.view(torch.int16)), f"rank {r}"


def test_ep_layer_one_rank_process_group_free():
    """No process group: ProcessGroupExchange is a single rank."""
    from layerstormexpertkernels_b200.ep import EPMoELayer
    w_gu, w_down, toks = _layer_setup(1, [150])
    bias = toks[0].bias.cuda()
    out = EPMoELayer(w_gu, w_down, bias, E_L, topk=K_L)(toks[0].hidden.cuda(),
                                                        toks[0].logits.cuda())
    ref = canonical_gpu(toks[0], w_gu, w_down, bias)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("tokens", [150, 1])
@pytest.mark.parametrize("combine", ["fused", "push"])
def test_ep_layer_peer_domain_one_rank(tokens, combine):
    """The peer-memory path (push dispatch; combine fused into the down GEMM
    epilogue, or a separate push kernel) with one rank, over three calls
    (three epochs)."""
    from layerstormexpertkernels_b200.ep import EPMoELayer, PeerDomain
    w_gu, w_down, toks = _layer_setup(1, [tokens])
    bias = toks[0].bias.cuda()
    with PeerDomain(max_tokens=512, hidden_dim=H_L, topk=K_L) as dom:
        layer = EPMoELayer(w_gu, w_down, bias, E_L, topk=K_L, domain=dom, combine=combine)
        ref = canonical_gpu(toks[0], w_gu, w_down, bias)
        for _ in range(3):
            out = layer(toks[0].hidden.cuda(), toks[0].logits.cuda())
            sync_and_check_device_error()
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert dom.epoch == 3


def test_peer_combine_push_one_rank():
    """Dispatch + combine without a GEMM (synthetic expert outputs, as the
    EP combine benchmark runs it) against the canonical per-slot combine."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200 import ep as EP
    T, E, H, k = 300, 64, 256, 8
    idx, w = _routing(T, E, k, seed=5, invalid=False)
    hidden = MO.bf16_round(np.random.default_rng(1).standard_normal((T, H), dtype=np.float32))
    with EP.PeerDomain(max_tokens=T, hidden_dim=H, topk=k) as dom:
        pd = EP.peer_dispatch(dom, bf16_dev(hidden), dev(idx), dev(w), E)
        permuted, offs, s2d, _ = P._C.ep_expert_permute(pd.recv_rows, pd.recv_ids, E,
                                                        pd.valid_slots)
        y = (permuted.float() * 1.5 + 0.25).to(torch.bfloat16)  # a row-wise "expert"
        out = EP.peer_combine(pd, y, s2d)
        sync_and_check_device_error()
    permuted1, offs1, s2d1, _ = P.moe_permute(bf16_dev(hidden), dev(idx), E)
    y1 = (permuted1.float() * 1.5 + 0.25).to(torch.bfloat16)
    ref = P.moe_combine_reduce_slots_bf16_to_bf16(
        P.moe_unpermute_bf16_perslot(y1, dev(w), s2d1, T, k))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("R,k,offset", [(1, 8, 0), (1023, 8, 0), (1025, 8, 1), (16384, 8, 0),
                                        (16385, 8, 0), (50000, 8, 1), (20000, 5, 0), (3, 1, 0)])
def test_slot_scan_sizes(R, k, offset):
    """The one-CTA slot scan across its pass boundary (16384 rows a pass),
    with 16-byte row loads (k = 8 on a 16-byte boundary) and scalar loads
    (other k, or a view that starts 4 bytes past the boundary)."""
    import layerstormexpertkernels_b200 as P
    rng = np.random.default_rng(R * 7 + k)
    ids = rng.integers(-1, 6, size=R * k + offset, dtype=np.int32)  # about 1 in 7 invalid
    view = dev(ids)[offset:].view(R, k)
    scan = P._C.ep_slot_scan(view)
    sync_and_check_device_error()
    assert np.array_equal(scan.cpu().numpy(), EO.ep_slot_scan(ids[offset:].reshape(R, k)))


def test_combine_plan_chunks_lists_every_row_once():
    """lsek_ep_combine_plan_chunks gives the plan of lsek_ep_combine_plan and
    chunk lists that hold every permuted row exactly once, each in the chunk
    of its source token (token // chunk_tokens, the last chunk taking the
    rest)."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200 import ep as EP
    T, E, H, k, C = 1000, 64, 64, 8, 3
    idx, w = _routing(T, E, k, seed=9)
    hidden = MO.bf16_round(np.random.default_rng(2).standard_normal((T, H), dtype=np.float32))
    with EP.PeerDomain(max_tokens=1024, hidden_dim=H, topk=k, combine_chunks=C) as dom:
        pd = EP.peer_dispatch(dom, bf16_dev(hidden), dev(idx), dev(w), E)
        permuted, _, s2d, _ = P._C.ep_expert_permute(pd.recv_rows, pd.recv_ids, E, pd.valid_slots)
        R, V = pd.recv_rows.shape[0], pd.valid_slots
        slot_row = P._C.ep_slot_scan(pd.recv_ids)
        plain = P._C.ep_combine_plan(dom.handle, s2d, slot_row, pd.counts, R, V)
        ct = -(-1024 // C)
        dr, drow, dw, order, count = P._C.ep_combine_plan_chunks(
            dom.handle, s2d, slot_row, pd.counts, R, V, ct, C)
        EP.peer_combine(pd, permuted, s2d)  # completes the epoch
        sync_and_check_device_error()
        ids = pd.recv_ids.cpu().numpy()
    assert torch.equal(dr, plain[0]) and torch.equal(drow, plain[1])
    assert torch.equal(dw.view(torch.int32), plain[2].view(torch.int32))
    assert pd.chunk_tokens == -(-T // C)  # the call's own chunks: T tokens on the one rank
    _, _, _, row_pair = P._C.ep_plan(dev(idx), E, 1)
    token = row_pair.cpu().numpy()[:R]
    p_of = s2d.cpu().numpy().reshape(R, k)
    want = np.full(V, -1)
    for r in range(R):
        for j in range(k):
            if ids[r, j] >= 0 and 0 <= p_of[r, j] < V:
                want[p_of[r, j]] = min(token[r] // ct, C - 1)
    assert (want >= 0).all()
    order, count = order.cpu().numpy().reshape(C, V), count.cpu().numpy()
    assert count.sum() == V
    seen = np.concatenate([order[c, :count[c]] for c in range(C)])
    assert np.array_equal(np.sort(seen), np.arange(V))
    for c in range(C):
        assert (want[order[c, :count[c]]] == c).all(), c


def test_peer_wait_expires_with_status():
    """A wait on an epoch nobody publishes gives up after its limit and
    records kDevErrEpDispatchWait (4); the context stays usable."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.ep import PeerDomain
    with PeerDomain(max_tokens=4, hidden_dim=64, topk=2) as dom:
        P._C.ep_wait(dom.handle, 0, 7, 2_000_000)  # 2 ms
        assert P.device_error() == 4
        P._C.ep_wait(dom.handle, 1, 7, 2_000_000)
        assert P.device_error() == 5
    x = torch.ones(4, device="cuda")
    assert float((x + 1).sum()) == 8.0
    assert P.device_error() == 0


@pytest.mark.parametrize("transport", ["nccl", "peer", "peer-push", "replicated"])
def test_ep_layer_two_gpus(tmp_path, transport):
    """Two processes (one GPU each), each checking its tokens against the
    one-GPU canonical path on its own GPU, over three calls."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = {"nccl": "29641", "peer": "29643", "peer-push": "29645", "replicated": "29647"}[transport]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", port,
           os.path.join(ROOT, "tests", "ep_nccl_worker.py"), str(tmp_path), transport]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(["timeout", "-k", "30", "600"] + cmd, cwd=ROOT, env=env,
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    for r in range(2):
        assert (tmp_path / f"ok{r}").read_text() == "bit-exact"


@pytest.mark.parametrize("transport", ["peer-push", "nccl"])
def test_ep_layer_two_gpus_cfg3_shape(tmp_path, transport):
    """The EP layer at the full cfg3 shape (T = 8192 tokens per rank, E = 256,
    H = 7168, I = 2048, top-8 of 8 groups / 4 kept) on two processes, each
    rank's output bit-identical to the one-GPU canonical path with all 256
    experts on its GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = {"peer-push": "29651", "nccl": "29653"}[transport]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", port,
           os.path.join(ROOT, "tests", "ep_nccl_worker.py"), str(tmp_path), transport, "cfg3"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(["timeout", "-k", "30", "900"] + cmd, cwd=ROOT, env=env,
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    for r in range(2):
        assert (tmp_path / f"ok{r}").read_text() == "bit-exact"


def test_copy_to_mapped_host():
    """The counts read used by the peer transport: a kernel stores through the
    pinned buffer's device mapping, even while a large device-to-host copy
    is queued on another stream."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200 import ep as EP
    src = torch.arange(40, dtype=torch.int32, device="cuda") * 3 - 7
    host = torch.zeros(40, dtype=torch.int32, pin_memory=True)
    big = torch.randn(64 << 20, device="cuda")
    big_h = torch.empty(big.shape, pin_memory=True)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        big_h.copy_(big, non_blocking=True)
    P._C.copy_to_mapped_host(host, src)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(host, src.cpu())
    side.synchronize()
    with pytest.raises(Exception):
        P._C.copy_to_mapped_host(torch.zeros(40, dtype=torch.int32), src)  # pageable
    mirror = EP.HostMirror()
    got = mirror.read(src.view(5, 8))
    assert got.shape == (5, 8) and torch.equal(got, src.view(5, 8).cpu())
