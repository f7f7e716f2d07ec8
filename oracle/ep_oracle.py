"""CPU restatement of the expert-parallel dispatch/combine steps.

TEST INFRASTRUCTURE ONLY: tests/ use it to check the EP kernels one by one
and, wrapped as a steps backend, to run the EP host logic over gloo on CPU.
The product never imports it.

The combine it defines is the reference's canonical per-slot combine
(moe_unpermute_bf16_perslot then moe_combine_reduce_slots_bf16_to_bf16,
smxx/permute/moe_permute.h:67-99 and moe_permute.cu:389-474; modelled in
tests/test_kernels.py:131-142, 187-200) split across ranks: ep_reference()
below composes the steps for all ranks at once and must equal
moe_oracle.reduce_slots(moe_oracle.moe_unpermute_perslot_bf16(...)) on the
same expert outputs, bit for bit.  The exchange layout (send rows per
destination in token order, combine rows in received-row and slot order) is
this build's own design; the reference has no EP exchange.

Arrays are numpy; bf16 payloads are fp32 arrays of exactly representable
bf16 values.
"""
from __future__ import annotations

import numpy as np

from . import moe_oracle as mo

F32 = np.float32


def owner(topk_indices, num_experts: int, world_size: int) -> np.ndarray:
    """Rank owning each slot's expert (-1 for an index outside [0, E))."""
    idx = np.asarray(topk_indices).astype(np.int64)
    per = num_experts // world_size
    return np.where((idx >= 0) & (idx < num_experts), idx // per, -1)


def ep_plan(topk_indices, num_experts: int, world_size: int):
    """(send_off [G+1], send_counts [G, 2], pair_row [T*G], row_pair [T*G]).

    Key of (t, g) = g when token t has an expert on rank g, else G; the
    stable sort of the keys orders the send rows rank-major and by token
    inside a rank (the moe_permute route with G 'experts')."""
    own = owner(topk_indices, num_experts, world_size)
    T = own.shape[0]
    G = world_size
    slots = np.stack([(own == g).sum(axis=1) for g in range(G)], axis=1) if T else \
        np.zeros((0, G), dtype=np.int64)
    keys = np.where(slots > 0, np.arange(G)[None, :], G).astype(np.int32)
    _, off, s2d, perm = mo.moe_permute(None, keys.reshape(T, G), G)
    counts = np.zeros((G, 2), dtype=np.int32)
    counts[:, 0] = np.diff(off)
    counts[:, 1] = slots.sum(axis=0)
    return off, counts, s2d, perm


def ep_dispatch_pack(hidden, topk_indices, topk_weights, pair_row, send_off, num_experts: int,
                     world_size: int):
    """(send_rows [rows, H], send_ids [rows, k], send_w [rows, k])."""
    idx = np.asarray(topk_indices)
    w = np.asarray(topk_weights, dtype=F32)
    T, k = idx.shape
    G, per = world_size, num_experts // world_size
    rows = int(send_off[G])
    own = owner(idx, num_experts, G)
    hid = np.asarray(hidden)
    send_rows = np.zeros((rows, hid.shape[1]), dtype=hid.dtype)
    send_ids = np.full((rows, k), -1, dtype=np.int32)
    send_w = np.zeros((rows, k), dtype=F32)
    pr = np.asarray(pair_row).reshape(T, G)
    for t in range(T):
        for g in range(G):
            r = pr[t, g]
            if r >= rows:
                continue
            send_rows[r] = hid[t]
            mine = own[t] == g
            send_ids[r] = np.where(mine, idx[t] - g * per, -1)
            send_w[r] = np.where(mine, w[t], F32(0))
    return send_rows, send_ids, send_w


def ep_slot_scan(ids) -> np.ndarray:
    """slot_row [rows+1]: exclusive scan of the valid (>= 0) ids per row."""
    valid = (np.asarray(ids) >= 0).sum(axis=1)
    return np.concatenate([[0], np.cumsum(valid)]).astype(np.int32)


def ep_expert_permute(rows_in, local_ids, local_experts: int):
    """(permuted [valid, H], offsets, s2d, perm): moe_permute with -1 as the
    sentinel, keeping only the valid slots' rows."""
    permuted, off, s2d, perm = mo.moe_permute(rows_in, local_ids, local_experts)
    nv = int(off[local_experts])
    return (None if permuted is None else permuted[:nv]), off, s2d, perm


def ep_combine_pack(expert_out, s2d, ids, weights, slot_row) -> np.ndarray:
    """Combine rows bf16(w * y[s2d]) of the valid slots, in row and slot order."""
    ids = np.asarray(ids)
    w = np.asarray(weights, dtype=F32)
    y = np.asarray(expert_out, dtype=F32)
    R, k = ids.shape
    d = np.asarray(s2d).reshape(R, k)
    comb = np.zeros((int(slot_row[R]), y.shape[1]), dtype=F32)
    for i in range(R):
        q = int(slot_row[i])
        for j in range(k):
            if ids[i, j] < 0:
                continue
            comb[q] = mo.bf16_round((w[i, j] * y[d[i, j]]).astype(F32))
            q += 1
    return comb


def ep_combine_reduce(comb_rows, topk_indices, pair_row, slot_row, num_experts: int,
                      world_size: int) -> np.ndarray:
    """out[t] = bf16(((0 + c[t,0]) + c[t,1]) + ...), c[t,j] the returned
    combine row of slot j (+0 for a slot without a valid expert)."""
    idx = np.asarray(topk_indices)
    T, k = idx.shape
    G = world_size
    own = owner(idx, num_experts, G)
    c = np.asarray(comb_rows, dtype=F32)
    H = c.shape[1] if c.ndim == 2 else 0
    pr = np.asarray(pair_row).reshape(T, G)
    acc = np.zeros((T, H), dtype=F32)
    for t in range(T):
        for j in range(k):
            g = own[t, j]
            if g < 0:
                acc[t] = (acc[t] + F32(0)).astype(F32)
                continue
            rank = int((own[t, :j] == g).sum())
            acc[t] = (acc[t] + c[int(slot_row[pr[t, g]]) + rank]).astype(F32)
    return mo.bf16_round(acc)


def ep_reference(hidden_per_rank, idx_per_rank, w_per_rank, num_experts: int, expert_fn):
    """All G ranks' EP layer composed in one process, with the exchanges
    done by slicing.  expert_fn(rank, permuted, offsets) -> y [valid, H].
    Returns the per-rank outputs [T_r, H]."""
    G = len(hidden_per_rank)
    El = num_experts // G
    plans, packs = [], []
    for r in range(G):
        off, counts, pair_row, _ = ep_plan(idx_per_rank[r], num_experts, G)
        plans.append((off, counts, pair_row))
        packs.append(ep_dispatch_pack(hidden_per_rank[r], idx_per_rank[r], w_per_rank[r],
                                      pair_row, off, num_experts, G))
    combs = []
    for g in range(G):
        parts = [(packs[r][0][plans[r][0][g]:plans[r][0][g + 1]],
                  packs[r][1][plans[r][0][g]:plans[r][0][g + 1]],
                  packs[r][2][plans[r][0][g]:plans[r][0][g + 1]]) for r in range(G)]
        rows = np.concatenate([p[0] for p in parts])
        ids = np.concatenate([p[1] for p in parts])
        wts = np.concatenate([p[2] for p in parts])
        permuted, off, s2d, _ = ep_expert_permute(rows, ids, El)
        y = expert_fn(g, permuted, off)
        slot_row = ep_slot_scan(ids)
        comb = ep_combine_pack(y, s2d, ids, wts, slot_row)
        # split back by source rank
        row_counts = [plans[r][1][g, 0] for r in range(G)]
        bounds = np.concatenate([[0], np.cumsum(row_counts)])
        combs.append([comb[slot_row[bounds[r]]:slot_row[bounds[r + 1]]] for r in range(G)])
    outs = []
    for r in range(G):
        back = np.concatenate([combs[g][r] for g in range(G)])
        send_slot_row = ep_slot_scan(packs[r][1])
        outs.append(ep_combine_reduce(back, idx_per_rank[r], plans[r][2], send_slot_row,
                                      num_experts, G))
    return outs
