"""GPU parity of the whole routed-expert layer (gating -> permute -> gate/up
GEMM + SwiGLU -> down GEMM -> weighted unpermute) against the oracle, at
small shapes in full and at DeepSeek-V3 shape on sampled tokens.  Routing is
bit-exact; outputs meet the layer bar of gpu_util.assert_layer_close."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_layer_close, sync_and_check_device_error
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


class StreamedExperts:
    """w[e] -> one expert's weights as fp32 numpy, copied from the GPU on
    demand (the full DeepSeek weight set is 22.5 GB)."""

    def __init__(self, t):
        self.t = t

    def __getitem__(self, e):
        return self.t[e].float().cpu().numpy()


def run_layer(x, w_gu, w_down, topk, n_group, topk_group, rsf=2.5, limit=0.0,
              scoring="sigmoid"):
    import layerstormexpertkernels_b200 as P
    out, w, idx = P.moe_layer_forward(x.hidden.cuda(), x.logits.cuda(), x.bias.cuda(), w_gu,
                                      w_down, topk, n_group, topk_group, rsf, True, scoring,
                                      limit, return_routing=True)
    sync_and_check_device_error()
    return out, w, idx


@pytest.mark.parametrize("T,E,H,I,k,ng,tg,limit,scoring", [
    (64, 16, 256, 128, 4, 4, 2, 0.0, "sigmoid"),
    (1, 16, 512, 256, 4, 1, 1, 0.0, "sigmoid"),
    (200, 32, 384, 96, 6, 8, 4, 10.0, "sqrtsoftplus"),
    (513, 8, 128, 64, 2, 1, 1, 0.0, "sigmoid"),
])
def test_layer_small_vs_oracle(T, E, H, I, k, ng, tg, limit, scoring):
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs
    x = token_inputs(T, E, H, seed=T + E)
    w_gu, w_down = expert_weights(E, H, I, device="cuda", seed_base=5000)
    out, w, idx = run_layer(x, w_gu, w_down, k, ng, tg, limit=limit, scoring=scoring)
    ref_bits, ow, oidx = O.moe_layer_forward(
        x.hidden.float().numpy(), x.logits.numpy(), x.bias.numpy(), StreamedExperts(w_gu),
        StreamedExperts(w_down), k, ng, tg, 2.5, True, scoring, limit)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.abs(w.cpu().numpy() - ow).max() <= 1e-6 * np.abs(ow).max()
    assert_layer_close(out, O.bf16_from_bits(ref_bits))


@pytest.mark.parametrize("T,sample", [(1, 1), (8, 4), (64, 3), (4096, 4)])
def test_layer_deepseek_shape_sampled(deepseek_weights, T, sample):
    """DeepSeek-V3 routed layer (E=256, H=7168, I=2048, top-8, 8 groups / 4
    kept).  Every token's output depends only on its own routing and experts,
    so a sample of tokens is checked against the oracle in full; each
    distinct expert is fetched to the host once."""
    from layerstormexpertkernels_b200.synthetic import token_inputs
    w_gu, w_down = deepseek_weights
    x = token_inputs(T, seed=T)
    out, w, idx = run_layer(x, w_gu, w_down, 8, 8, 4)
    ow, oidx = O.topk_gating(x.logits.numpy(), x.bias.numpy(), 8, 8, 4, 2.5, True)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    rng = np.random.default_rng(T)
    toks = np.sort(rng.choice(T, size=sample, replace=False))
    hidden = x.hidden.float().numpy()
    y = np.zeros((len(toks), 8, hidden.shape[1]), np.float32)
    for e in sorted(set(oidx[toks].ravel().tolist())):
        gu = w_gu[e].float().cpu().numpy()
        gd = w_down[e].float().cpu().numpy()
        for i, t in enumerate(toks):
            for j in np.nonzero(oidx[t] == e)[0]:
                y[i, j] = O.expert_ffn(hidden[t:t + 1], gu, gd)[0]
    refs = [O.bf16_from_bits(O.moe_unpermute(O.bf16_bits(y[i]), ow[t:t + 1],
                                             np.arange(8, dtype=np.int32), 1, 8))
            for i, t in enumerate(toks)]
    assert_layer_close(out[torch.as_tensor(toks).cuda()], np.concatenate(refs))


# Experts with crafted row counts at cfg1 and the GEMM unit kinds each one
# exercises (tiles are 128 rows; 256-row blocks run as paired units; the
# rows after them: more than 192 as a pair of up to 256, 129..192 as one
# wide swapped tile, at most 128 as one tile; at most 64 rows after a block
# turn that block's second half and them into one wide tile).
TILE_CLASS_COUNTS = {
    3: 1,       # one tile with one valid row
    5: 520,     # a paired unit, a full tile and a wide tile of 136 rows
    9: 64,      # one tile of 64 rows
    12: 255,    # a paired unit whose second tile has 127 rows
    17: 65,     # one tile of 65 rows
    25: 192,    # one wide swapped tile at its largest width (N = 192)
    26: 193,    # a paired unit whose second tile has 65 rows
    30: 128,    # one full tile
    33: 129,    # one wide swapped tile of 129 rows (N = 144)
    40: 256,    # a paired unit of two full tiles
    47: 300,    # a full tile + a wide tile of 172 rows
    50: 400,    # a paired unit + a wide tile of 144 rows
    55: 356,    # a paired unit + a 100-row tile
    62: 1100,   # the heaviest expert: four paired units + a 76-row tile
}
# Partners for the probe tokens' remaining slots (groups 2 and 3), so the
# oracle needs the weights of only these and the special experts.
PROBE_MATES = (69, 78, 87, 95, 98, 107, 116, 125)


def _tile_boundary_ranks(count):
    ranks = {0, count - 1}
    for b in (63, 64, 127, 128, 255, 256, 511, 512, 1023, 1024):
        if b < count:
            ranks.add(b)
    return ranks


def craft_tile_class_routing(T=4096, E=256, k=8, n_group=8, seed=11):
    """Per-token expert sets for which the special experts receive exactly
    TILE_CLASS_COUNTS rows, each token's experts lie in at most four of the
    eight groups, and the tokens at every tile-boundary rank of a special
    expert ("probes") take their other slots from PROBE_MATES.  A token's
    rank inside an expert is its position in token order (the permute is a
    stable sort of t * k + slot).  Returns (sets [T] of lists, probe tokens)."""
    rng = np.random.default_rng(seed)
    epg = E // n_group
    special = list(TILE_CLASS_COUNTS)
    excluded = set(special) | set(PROBE_MATES)
    taken = {e: 0 for e in special}
    ranks = {e: _tile_boundary_ranks(c) for e, c in TILE_CLASS_COUNTS.items()}
    sets, probes = [], []
    for t in range(T):
        left = T - t
        joined, probe = [], False
        for e in rng.permutation(special):
            need = TILE_CLASS_COUNTS[e] - taken[e]
            if need > 0 and (need >= left or rng.random() < need / left):
                assert len(joined) < k, "routing construction ran out of slots"
                probe |= taken[e] in ranks[e]
                taken[e] += 1
                joined.append(int(e))
        if probe:
            fill = [m for m in PROBE_MATES][: k - len(joined)]
        else:
            groups = {e // epg for e in joined}
            while len(groups) < 4:
                groups.add(int(rng.integers(n_group)))
            pool = [e for g in sorted(groups) for e in range(g * epg, (g + 1) * epg)
                    if e not in excluded]
            fill = [int(e) for e in rng.choice(pool, size=k - len(joined), replace=False)]
        sets.append(joined + fill)
        if probe:
            probes.append(t)
    assert all(taken[e] == c for e, c in TILE_CLASS_COUNTS.items())
    return sets, probes


def test_layer_cfg1_every_tile_class_vs_oracle(deepseek_weights):
    """cfg1 layer (T=4096) on crafted logits: experts with 1, 64, 65, 128,
    129, 192, 193, 255, 256, 300, 356, 400, 520 and 1100 rows, so every GEMM
    unit kind of both projections occurs (single full and partial tiles,
    wide swapped tiles from N=144 to N=192 alone, after a pair and after a
    split block, paired units with full and partial second tiles, the
    heaviest expert's tail).  The tokens sitting at every
    tile-boundary row of those experts are checked in full against the oracle
    (all 7168 columns cross every n-tile of the down projection)."""
    from layerstormexpertkernels_b200.synthetic import token_inputs
    w_gu, w_down = deepseek_weights
    T, E, H, k = 4096, 256, 7168, 8
    sets, probes = craft_tile_class_routing(T, E, k)
    x = token_inputs(T, seed=4242)
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal((T, E)) * 0.5 - 8.0).astype(np.float32)
    for t, s in enumerate(sets):
        logits[t, s] = (4.0 + 0.5 * rng.random(len(s))).astype(np.float32)
    x.logits = torch.from_numpy(logits)
    out, w, idx = run_layer(x, w_gu, w_down, 8, 8, 4)
    ow, oidx = O.topk_gating(logits, x.bias.numpy(), 8, 8, 4, 2.5, True)
    gidx = idx.cpu().numpy()
    assert np.array_equal(gidx, oidx)
    assert np.abs(w.cpu().numpy() - ow).max() <= 1e-6 * np.abs(ow).max()
    assert all(set(oidx[t].tolist()) == set(s) for t, s in enumerate(sets))
    counts = np.bincount(oidx.ravel(), minlength=E)
    for e, c in TILE_CLASS_COUNTS.items():
        assert counts[e] == c
    assert counts.argmax() == 62
    toks = np.array(probes)
    hidden = x.hidden.float().numpy()
    y = np.zeros((len(toks), k, H), np.float32)
    for e in sorted(set(oidx[toks].ravel().tolist())):
        rows = [(i, j) for i, t in enumerate(toks) for j in np.nonzero(oidx[t] == e)[0]]
        ye = O.expert_ffn(hidden[[toks[i] for i, _ in rows]], w_gu[e].float().cpu().numpy(),
                          w_down[e].float().cpu().numpy())
        for r, (i, j) in enumerate(rows):
            y[i, j] = ye[r]
    refs = [O.bf16_from_bits(O.moe_unpermute(O.bf16_bits(y[i]), ow[t:t + 1],
                                             np.arange(k, dtype=np.int32), 1, k))
            for i, t in enumerate(toks)]
    assert_layer_close(out[torch.as_tensor(toks).cuda()], np.concatenate(refs))


def test_layer_class_reuses_workspace(deepseek_weights):
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import token_inputs
    w_gu, w_down = deepseek_weights
    layer = P.MoELayer(w_gu, w_down, token_inputs(1).bias.cuda(), max_tokens=64)
    ws = layer.workspace.data_ptr()
    x = token_inputs(64, seed=3)
    a = layer(x.hidden.cuda(), x.logits.cuda())
    b = layer(x.hidden.cuda(), x.logits.cuda())
    sync_and_check_device_error()
    assert layer.workspace.data_ptr() == ws
    assert torch.equal(a, b)  # deterministic


@pytest.fixture(scope="module")
def deepseek_weights():
    from layerstormexpertkernels_b200.synthetic import expert_weights
    w = expert_weights(device="cuda")
    yield w
    del w
    torch.cuda.empty_cache()


def test_host_pipeline_matches_direct_calls():
    """HostPipeline (copies on their own streams, two device buffer sets)
    gives each batch the output of a direct call on that batch."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs
    T, E, H, I = 96, 16, 256, 128
    w_gu, w_down = expert_weights(E, H, I, device="cuda", seed_base=9000)
    bias = token_inputs(1, E, 8, seed=3).bias.cuda()
    layer = P.MoELayer(w_gu, w_down, bias, topk=4, n_group=4, topk_group=2)
    batches = [token_inputs(T, E, H, seed=50 + i) for i in range(5)]
    ins = [(b.hidden.pin_memory(), b.logits.pin_memory()) for b in batches]
    outs = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in batches]
    pipe = P.HostPipeline(lambda h, l: layer(h, l), (T, H), (T, E), torch.device("cuda"))
    for (h, l), o in zip(ins, outs):
        pipe.submit(h, l, o)
    pipe.synchronize()
    sync_and_check_device_error()
    for b, o in zip(batches, outs):
        ref = layer(b.hidden.cuda(), b.logits.cuda()).cpu()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("T_small", [1, 7, 32])
def test_decode_geometry_matches_full_geometry(deepseek_weights, T_small):
    """T <= 32 runs the GEMMs with the decode pipeline geometry (32-row token
    box, six stages); a token's output depends only on its own routing, so
    the first tokens of a larger call (full geometry) must have the same
    bits."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import token_inputs
    w_gu, w_down = deepseek_weights
    x = token_inputs(80, 256, 7168, seed=77)
    bias = x.bias.cuda()
    big = P.moe_layer_forward(x.hidden.cuda(), x.logits.cuda(), bias, w_gu, w_down, 8, 8, 4, 2.5,
                              True)
    small = P.moe_layer_forward(x.hidden[:T_small].cuda(), x.logits[:T_small].cuda(), bias, w_gu,
                                w_down, 8, 8, 4, 2.5, True)
    sync_and_check_device_error()
    assert torch.equal(small.view(torch.int16), big[:T_small].view(torch.int16))


@pytest.mark.parametrize("T_small", [16, 64])
def test_gathered_rows_match_copied_rows(deepseek_weights, T_small):
    """Up to 64 tokens the layer gathers the token rows inside the gate/up
    GEMM (TMA gather of four rows); larger calls copy them first.  Same bits
    for the tokens both calls share."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import token_inputs
    w_gu, w_down = deepseek_weights
    x = token_inputs(160, 256, 7168, seed=91)
    bias = x.bias.cuda()
    big = P.moe_layer_forward(x.hidden.cuda(), x.logits.cuda(), bias, w_gu, w_down, 8, 8, 4, 2.5,
                              True)
    small = P.moe_layer_forward(x.hidden[:T_small].cuda(), x.logits[:T_small].cuda(), bias, w_gu,
                                w_down, 8, 8, 4, 2.5, True)
    sync_and_check_device_error()
    assert torch.equal(small.view(torch.int16), big[:T_small].view(torch.int16))


def test_bind_host_to_device():
    import os

    import layerstormexpertkernels_b200 as P
    before = os.sched_getaffinity(0)
    try:
        cores = P.bind_host_to_device(torch.device("cuda", 0))
        if cores is not None:
            assert cores and set(cores) <= before
            assert os.sched_getaffinity(0) == set(cores)
    finally:
        os.sched_setaffinity(0, before)


@pytest.mark.parametrize("T", [1, 64, 300])
def test_layer_replays_from_a_cuda_graph(T):
    """The layer launches nothing that a CUDA graph cannot hold: captured once
    (workspace and outputs preallocated), a replay on new inputs written into
    the same buffers gives the bits of an eager call.  T=1 / 64 take the
    decode and gathered paths, 300 the row copy."""
    import layerstormexpertkernels_b200 as P
    from layerstormexpertkernels_b200.synthetic import expert_weights, token_inputs
    E, H, I = 32, 1024, 512
    w_gu, w_down = expert_weights(E, H, I, device="cuda", seed_base=4000)
    x0, x1 = token_inputs(T, E, H, seed=T), token_inputs(T, E, H, seed=T + 1)
    layer = P.MoELayer(w_gu, w_down, x0.bias.cuda(), topk=8, n_group=8, topk_group=4,
                       max_tokens=T)
    hidden, logits = x0.hidden.cuda(), x0.logits.cuda()
    out = torch.empty_like(hidden)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            layer(hidden, logits, out=out)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer(hidden, logits, out=out)
    hidden.copy_(x1.hidden.cuda())
    logits.copy_(x1.logits.cuda())
    graph.replay()
    torch.cuda.synchronize()
    sync_and_check_device_error()
    ref = layer(x1.hidden.cuda(), x1.logits.cuda())
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    del graph
