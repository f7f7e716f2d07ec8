"""Expert-parallel MoE layer: experts sharded over the ranks of a process
group, tokens exchanged either with two NCCL all-to-alls or through peer
memory over NVLink (`PeerDomain`: the dispatch and combine kernels store
straight into the owner's buffers, epoch flags order them).

Rank g of G owns experts [g*E/G, (g+1)*E/G).  Per layer:

  1. gate locally (topk_gating on this rank's tokens);
  2. plan: a stable counting sort of (token, destination rank) pairs gives
     each destination's send rows in token order, and per destination the
     number of rows and of (token, slot) pairs it serves; the [G, 2] counts
     are exchanged once and read by the host once (the only host
     synchronisation of the layer);
  3. dispatch: each token row once per distinct owner rank, with per slot
     the expert's local index (-1 for other ranks' experts) and weight;
  4. expert side: permute the received rows by local expert (only own
     slots are copied), gate/up GEMM with fused SwiGLU, down GEMM, then the
     weighted per-slot pack bf16(w * y) in received-row and slot order;
  5. combine: the packed slots go back (the reverse all-to-all, or a push
     into the source rank's combine buffer);
  6. the source rank sums each token's slots in slot order in fp32 from 0
     and rounds once to bf16 (over peer memory, per token chunk as soon as
     every rank has pushed that chunk, beside the later chunks' pushes).

Steps 4-6 reproduce moe_unpermute_bf16_perslot followed by
moe_combine_reduce_slots_bf16_to_bf16 (smxx/permute/moe_permute.h:67-99 of
the reference) bit for bit, for every world size: the per-slot product and
the fixed-order sum are the same operations on the same values.  The
reference leaves the exchange to its consumer and models it as an
all-reduce of [T, topk, H] (tests/test_kernels.py:131-142, 187-200); only
the rows that cross ranks travel here.

Every data-path step is a CUDA kernel of liblsek.so (`DeviceSteps`); the
NCCL transport's collectives are torch.distributed all_to_all_single calls
(`ProcessGroupExchange`).  Both can be replaced: the CPU tests inject a
restatement of the kernels to check this module's exchange logic over gloo,
and the one-GPU tests run G ranks as threads with an in-process exchange.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _C


class DeviceSteps:
    """The device kernels of each EP step (liblsek.so through the binding)."""

    plan = staticmethod(_C.ep_plan)
    dispatch_pack = staticmethod(_C.ep_dispatch_pack)
    slot_scan = staticmethod(_C.ep_slot_scan)
    expert_permute = staticmethod(_C.ep_expert_permute)
    combine_pack = staticmethod(_C.ep_combine_pack)
    combine_reduce = staticmethod(_C.ep_combine_reduce)
    topk_gating = staticmethod(_C.topk_gating)
    grouped_gemm_swiglu = staticmethod(_C.grouped_gemm_swiglu_bf16)
    grouped_gemm = staticmethod(_C.grouped_gemm_bf16)
    moe_permute = staticmethod(_C.moe_permute)
    unpermute_perslot = staticmethod(_C.moe_unpermute_bf16_perslot)
    reduce_slots = staticmethod(_C.moe_combine_reduce_slots_bf16_to_bf16)


def _as_words(t: torch.Tensor) -> torch.Tensor:
    """A 2-D tensor viewed as 32-bit words (bf16 rows travel as int32 pairs,
    which every backend moves bit for bit)."""
    if t.dtype in (torch.int32, torch.float32):
        return t
    return t.view(torch.int32)


class ProcessGroupExchange:
    """The exchange over a torch.distributed process group (NCCL on GPUs,
    gloo on CPU); with no initialised group it is a single rank."""

    def __init__(self, group=None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world_size, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world_size, self.rank = 1, 0

    def all_to_all(self, send: torch.Tensor, send_splits: list[int],
                   recv_splits: list[int]) -> torch.Tensor:
        """Variable all-to-all along dim 0; identity when there is one rank."""
        if self.world_size == 1:
            return send
        recv = send.new_empty((sum(recv_splits),) + tuple(send.shape[1:]))
        dist.all_to_all_single(_as_words(recv), _as_words(send), output_split_sizes=recv_splits,
                               input_split_sizes=send_splits, group=self.group)
        return recv

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        """In-place SUM over the ranks.  bf16 reduces natively on GPUs; on
        the CPU (gloo) it goes through fp32, which is exact for the sums of
        one value and zeros this module uses it for."""
        if self.world_size == 1:
            return t
        if t.is_cuda or t.dtype != torch.bfloat16:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            return t
        f = t.float()
        dist.all_reduce(f, op=dist.ReduceOp.SUM, group=self.group)
        t.copy_(f)
        return t


def as_exchange(group):
    """`group` may be None (the default process group, or one rank without
    one), a torch.distributed process group, or any object with world_size,
    rank and all_to_all(send, send_splits, recv_splits)."""
    if hasattr(group, "all_to_all"):
        return group
    return ProcessGroupExchange(group)


@dataclass
class Dispatch:
    """State of one dispatch, needed again by the combine.

    Sender side: the token routing, the plan and the sent slot ids.
    Expert side: the received rows, local ids and weights, and the split
    sizes of both exchanges (host ints)."""

    num_tokens: int
    num_experts: int
    world_size: int
    topk_indices: torch.Tensor          # [T, k] this rank's routing
    pair_row: torch.Tensor              # [T*G] send row of (token, rank)
    send_ids: torch.Tensor              # [rows, k] local ids at the destination
    send_rows_n: list[int]              # rows sent to each rank
    send_slots_n: list[int]             # (token, slot) pairs served by each rank
    recv_rows: torch.Tensor             # [R, H] bf16
    recv_ids: torch.Tensor              # [R, k] int32, -1 = another rank's expert
    recv_w: torch.Tensor                # [R, k] fp32, 0 there
    recv_rows_n: list[int]
    recv_slots_n: list[int]

    @property
    def valid_slots(self) -> int:
        return sum(self.recv_slots_n)


# ---------------------------------------------------------------------------
# Peer-memory transport: the kernels move the data over NVLink themselves
# ---------------------------------------------------------------------------


class PeerDomain:
    """The symmetric buffers of an expert-parallel group on one node.

    Every rank allocates one buffer (liblsek lsek_ep_domain_create), the
    ranks swap its CUDA IPC handle over the process group once, and the
    dispatch / combine kernels then store straight into the owner's buffer.
    `max_tokens` bounds the tokens of one rank per layer call.  The combine
    runs in `combine_chunks` token chunks of ceil(T / combine_chunks) tokens,
    T the largest token count of any rank in that call (the same chunks on
    every rank): a rank reduces chunk c's tokens as soon as every rank has
    pushed its rows for them, while later chunks are still in flight.  close() (or leaving a `with` block) frees the buffers after a
    barrier, so no peer still writes into them."""

    def __init__(self, max_tokens: int, hidden_dim: int, topk: int, group=None,
                 combine_chunks: int = 4):
        ex = ProcessGroupExchange(group)
        self.group, self.world_size, self.rank = group, ex.world_size, ex.rank
        self.max_tokens, self.hidden_dim, self.topk = max_tokens, hidden_dim, topk
        self.combine_chunks = max(1, min(int(combine_chunks), 16, max(max_tokens, 1)))
        self._reduce_stream = None
        self._push_stream = None
        self.handle = _C.ep_domain_create(self.rank, self.world_size, max_tokens, hidden_dim, topk)
        try:
            if self.world_size > 1:
                mine = _C.ep_domain_export(self.handle)
                dev = torch.device("cuda", torch.cuda.current_device())
                every = torch.empty(self.world_size * mine.numel(), dtype=torch.uint8, device=dev)
                dist.all_gather_into_tensor(every, mine.to(dev), group=group)
                every = every.view(self.world_size, -1).cpu()
                for g in range(self.world_size):
                    if g != self.rank:
                        _C.ep_domain_import(self.handle, g, every[g].contiguous())
                dist.barrier(group=group)
        except BaseException:
            _C.ep_domain_destroy(self.handle)
            self.handle = 0
            raise
        (self.recv_rows, self.recv_ids, self.recv_w,
         self.back) = _C.ep_domain_buffers(self.handle, hidden_dim, topk)
        self.epoch = 0
        self.mirror = HostMirror()

    def reduce_stream(self) -> torch.cuda.Stream:
        if self._reduce_stream is None:
            self._reduce_stream = torch.cuda.Stream(device=torch.cuda.current_device())
        return self._reduce_stream

    def push_stream(self) -> torch.cuda.Stream:
        """A high-priority stream for combine pushes: the reduces that overlap
        them (on reduce_stream) then fill the SMs only behind the pushes'
        CTAs, which keep the NVLink stores in flight."""
        if self._push_stream is None:
            self._push_stream = torch.cuda.Stream(device=torch.cuda.current_device(),
                                                  priority=-1)
        return self._push_stream

    def next_epoch(self) -> int:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        return self.epoch

    def close(self):
        if self.handle:
            torch.cuda.synchronize()
            if self.world_size > 1:
                dist.barrier(group=self.group)
            self.recv_rows = self.recv_ids = self.recv_w = self.back = None
            _C.ep_domain_destroy(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@dataclass
class PeerDispatch:
    """One dispatch over a PeerDomain, needed again by the combine."""

    domain: PeerDomain
    epoch: int
    counts: torch.Tensor        # [G, G, 2] host: (rows, slots) rank s sends to rank g
    num_experts: int
    topk_indices: torch.Tensor
    pair_row: torch.Tensor
    send_ids: torch.Tensor
    recv_rows: torch.Tensor     # views of the domain's receive buffers
    recv_ids: torch.Tensor
    recv_w: torch.Tensor
    chunk_tokens: int           # combine chunk size of this call, the same on every rank

    @property
    def valid_slots(self) -> int:
        return int(self.counts[:, self.domain.rank, 1].sum())

    @property
    def back_rows(self) -> int:
        return int(self.counts[self.domain.rank, :, 1].sum())


class HostMirror:
    """Reads a small int32 device tensor into pinned host memory through a
    kernel (lsek_copy_to_mapped_host) instead of a copy-engine transfer, so
    the read never queues behind a large device-to-host copy of the previous
    batch's output on another stream (HostPipeline)."""

    def __init__(self):
        self.buf = None
        self.done = None

    def read(self, src: torch.Tensor) -> torch.Tensor:
        n = src.numel()
        if self.buf is None or self.buf.numel() < n:
            self.buf = torch.empty(n, dtype=torch.int32, pin_memory=True)
            self.done = torch.cuda.Event()
        host = self.buf[:n]
        _C.copy_to_mapped_host(host, src.reshape(-1).contiguous())
        self.done.record()
        self.done.synchronize()
        return host.clone().view(src.shape)


def _gather_counts(send_counts: torch.Tensor, domain: PeerDomain, num_tokens: int):
    """([G, G, 2] counts of every rank, the largest token count of any rank)
    on the host, from one all-gather of each rank's [G, 2] counts and its
    token count."""
    G = domain.world_size
    if G == 1:
        return domain.mirror.read(send_counts.reshape(1, 1, 2)), num_tokens
    mine = torch.cat([send_counts.reshape(-1),
                      torch.full((1,), num_tokens, dtype=torch.int32, device=send_counts.device)])
    every = torch.empty(G * (2 * G + 1), dtype=torch.int32, device=send_counts.device)
    dist.all_gather_into_tensor(every, mine, group=domain.group)
    host = domain.mirror.read(every.view(G, 2 * G + 1))
    return host[:, :2 * G].contiguous().view(G, G, 2), int(host[:, 2 * G].max())


def peer_dispatch(domain: PeerDomain, hidden: torch.Tensor, topk_indices: torch.Tensor,
                  topk_weights: torch.Tensor, num_experts: int, steps=DeviceSteps,
                  mark: Optional[Callable[[str], None]] = None) -> PeerDispatch:
    """Plan, then push every token row into its expert ranks' receive
    buffers and wait (bounded) for every rank's rows."""
    G, me = domain.world_size, domain.rank
    send_off, send_counts, pair_row, _ = steps.plan(topk_indices, num_experts, G)
    counts, t_max = _gather_counts(send_counts, domain, topk_indices.shape[0])
    if mark:
        mark("ep_plan")
    # The combine's token chunks cover the largest rank's tokens (at most
    # max_tokens), so every chunk holds tokens when the ranks are balanced.
    chunk_tokens = -(-max(min(t_max, domain.max_tokens), 1) // domain.combine_chunks)
    epoch = domain.next_epoch()
    rows = int(counts[me, :, 0].sum())
    send_ids = _C.ep_dispatch_push(domain.handle, counts, hidden, topk_indices, topk_weights,
                                   pair_row, send_off, rows, num_experts, epoch)
    if mark:
        mark("ep_dispatch_push")
    _C.ep_wait(domain.handle, 0, epoch)
    if mark:
        mark("ep_dispatch_wait")
    R = int(counts[:, me, 0].sum())
    return PeerDispatch(domain, epoch, counts, num_experts, topk_indices, pair_row, send_ids,
                        domain.recv_rows[:R], domain.recv_ids[:R], domain.recv_w[:R],
                        chunk_tokens)


def peer_combine_plan(pd: PeerDispatch, src_to_dest_map: torch.Tensor, steps=DeviceSteps):
    """(dst_rank, dst_row, dst_w) of every permuted row of the received slots."""
    slot_row = steps.slot_scan(pd.recv_ids)
    return _C.ep_combine_plan(pd.domain.handle, src_to_dest_map, slot_row, pd.counts,
                              pd.recv_rows.shape[0], pd.valid_slots)


def peer_combine_finish(pd: PeerDispatch, steps=DeviceSteps,
                        mark: Optional[Callable[[str], None]] = None) -> torch.Tensor:
    """Waits (bounded) for every rank's combine rows, then the fixed-order
    slot reduce of this rank's tokens."""
    _C.ep_wait(pd.domain.handle, 1, pd.epoch)
    if mark:
        mark("ep_combine_wait")
    send_slot_row = steps.slot_scan(pd.send_ids)
    out = steps.combine_reduce(pd.domain.back[:pd.back_rows], pd.topk_indices, pd.pair_row,
                               send_slot_row, pd.num_experts, pd.domain.world_size)
    if mark:
        mark("ep_combine_reduce")
    return out


def peer_combine_plan_chunked(pd: PeerDispatch, src_to_dest_map: torch.Tensor,
                              steps=DeviceSteps):
    """peer_combine_plan plus the rows of every token chunk, in one kernel
    (lsek_ep_combine_plan_chunks): (dst_rank, dst_row, dst_w, order,
    order_count), chunk c's rows being order[c * valid_slots :][:order_count[c]]."""
    dom = pd.domain
    slot_row = steps.slot_scan(pd.recv_ids)
    return _C.ep_combine_plan_chunks(dom.handle, src_to_dest_map, slot_row, pd.counts,
                                     pd.recv_rows.shape[0], pd.valid_slots, pd.chunk_tokens,
                                     dom.combine_chunks)


def peer_combine_chunked(pd: PeerDispatch, push_chunk: Callable[[int], None],
                         push_stream: torch.cuda.Stream, steps=DeviceSteps,
                         mark: Optional[Callable[[str], None]] = None) -> torch.Tensor:
    """The combine in token chunks: push_chunk(c) enqueues, on push_stream,
    the push of every row whose source token lies in chunk c and publishes
    chunk c (lsek_ep_combine_push_chunk).  On the domain's reduce stream,
    chunk c's reduce waits for that push (a stream event: the reduce never
    spins on a kernel of its own GPU) and, bounded, for every other rank's
    chunk-c flag, then sums its tokens' slots in fixed order; it overlaps the
    pushes of the later chunks.  Returns the [T, H] bf16 output (bit-identical
    to the unchunked combine: the same per-token sums)."""
    dom = pd.domain
    C, ct = dom.combine_chunks, pd.chunk_tokens
    T = pd.topk_indices.shape[0]
    G = dom.world_size
    main = torch.cuda.current_stream()
    red = dom.reduce_stream()
    out = torch.empty(T, dom.hidden_dim, dtype=torch.bfloat16, device=pd.topk_indices.device)
    back = dom.back[:pd.back_rows]
    pair_row = pd.pair_row.view(max(T, 1), G) if T > 0 else pd.pair_row.view(0, G)
    ready = torch.cuda.Event()
    ready.record(main)
    push_stream.wait_event(ready)
    red.wait_event(ready)
    with torch.cuda.stream(red):  # runs beside the first push
        send_slot_row = steps.slot_scan(pd.send_ids)
    for c in range(C):
        push_chunk(c)
        pushed = torch.cuda.Event()
        pushed.record(push_stream)
        red.wait_event(pushed)
        t0, t1 = min(c * ct, T), min((c + 1) * ct, T)
        with torch.cuda.stream(red):
            _C.ep_wait(dom.handle, 2 + c, pd.epoch)
            if t1 > t0:
                steps.combine_reduce(back, pd.topk_indices[t0:t1], pair_row[t0:t1], send_slot_row,
                                     pd.num_experts, G, out=out[t0:t1])
    if mark:
        main.wait_stream(push_stream)
        mark("ep_combine_push")
    main.wait_stream(red)
    if mark:
        mark("ep_combine_reduce")
    return out


def peer_combine(pd: PeerDispatch, expert_out: torch.Tensor, src_to_dest_map: torch.Tensor,
                 steps=DeviceSteps, mark: Optional[Callable[[str], None]] = None) -> torch.Tensor:
    """The weighted combine of expert outputs already in memory
    ([valid_slots, H] in the order of src_to_dest_map), pushed and reduced
    in token chunks (peer_combine_chunked)."""
    dom = pd.domain
    push = dom.push_stream()
    start = torch.cuda.Event()
    start.record(torch.cuda.current_stream())
    push.wait_event(start)
    with torch.cuda.stream(push):
        dst_rank, dst_row, dst_w, order, count = peer_combine_plan_chunked(pd, src_to_dest_map,
                                                                           steps)

    def push_chunk(c):
        with torch.cuda.stream(push):
            _C.ep_combine_push_chunk(dom.handle, expert_out, dst_rank, dst_row, dst_w, order,
                                     count, c, pd.epoch)

    return peer_combine_chunked(pd, push_chunk, push, steps, mark)


def dispatch(hidden: torch.Tensor, topk_indices: torch.Tensor, topk_weights: torch.Tensor,
             num_experts: int, group=None, steps=DeviceSteps,
             mark: Optional[Callable[[str], None]] = None) -> Dispatch:
    """Sends each token row to every rank that owns one of its experts.
    `mark(name)` (optional) is called after each phase, e.g. to record
    timing events."""
    ex = as_exchange(group)
    world = ex.world_size
    T, k = topk_indices.shape
    send_off, send_counts, pair_row, _ = steps.plan(topk_indices, num_experts, world)
    recv_counts = ex.all_to_all(send_counts, [1] * world, [1] * world)
    counts = torch.cat([send_counts.reshape(-1), recv_counts.reshape(-1)]).cpu().tolist()
    send_rows_n, send_slots_n = counts[0:2 * world:2], counts[1:2 * world:2]
    recv_rows_n, recv_slots_n = counts[2 * world::2], counts[2 * world + 1::2]
    if mark:
        mark("ep_plan")
    send_rows, send_ids, send_w = steps.dispatch_pack(hidden, topk_indices, topk_weights, pair_row,
                                                      send_off, sum(send_rows_n), num_experts,
                                                      world)
    if mark:
        mark("ep_dispatch_pack")
    recv_rows = ex.all_to_all(send_rows, send_rows_n, recv_rows_n)
    recv_ids = ex.all_to_all(send_ids, send_rows_n, recv_rows_n)
    recv_w = ex.all_to_all(send_w, send_rows_n, recv_rows_n)
    if mark:
        mark("ep_dispatch_exchange")
    return Dispatch(T, num_experts, world, topk_indices, pair_row, send_ids, send_rows_n,
                    send_slots_n, recv_rows, recv_ids, recv_w, recv_rows_n, recv_slots_n)


def combine(d: Dispatch, expert_out: torch.Tensor, src_to_dest_map: torch.Tensor, group=None,
            steps=DeviceSteps, mark: Optional[Callable[[str], None]] = None) -> torch.Tensor:
    """Weighted combine of the expert outputs back onto the source tokens.

    `expert_out` [valid_slots, H] bf16 holds the expert-side rows in the
    order of `src_to_dest_map` (the map returned by expert_permute)."""
    slot_row = steps.slot_scan(d.recv_ids)
    comb = steps.combine_pack(expert_out, src_to_dest_map, d.recv_ids, d.recv_w, slot_row,
                              d.valid_slots)
    if mark:
        mark("ep_combine_pack")
    back = as_exchange(group).all_to_all(comb, d.recv_slots_n, d.send_slots_n)
    if mark:
        mark("ep_combine_exchange")
    send_slot_row = steps.slot_scan(d.send_ids)
    out = steps.combine_reduce(back, d.topk_indices, d.pair_row, send_slot_row, d.num_experts,
                               d.world_size)
    if mark:
        mark("ep_combine_reduce")
    return out


def expert_permute(d: Dispatch, local_experts: int, steps=DeviceSteps):
    """Expert-major order of this rank's received slots:
    (permuted [valid_slots, H], offsets [local_experts+1], src_to_dest_map)."""
    permuted, offsets, s2d, _ = steps.expert_permute(d.recv_rows, d.recv_ids, local_experts,
                                                     d.valid_slots)
    return permuted, offsets, s2d


class EPMoELayer:
    """The routed-expert MoE layer with this rank's share of the experts.

    `w_gu` [E/G, 2I, H] and `w_down` [E/G, H, I] are the local experts'
    weights (gate rows first, as grouped_gemm_swiglu_bf16 expects); `bias` is
    the full [E] correction bias.  forward(hidden [T, H] bf16, logits [T, E]
    fp32) returns this rank's [T, H] bf16 layer output.

    With a PeerDomain the exchanges run over peer memory: the dispatch
    kernel stores rows into the owner ranks, and the weighted slots go back
    through a push kernel (combine="push", the default) or straight from the
    down-projection GEMM's epilogue (combine="fused").  Without a domain
    they are NCCL all-to-alls through `group`."""

    def __init__(self, w_gu: torch.Tensor, w_down: torch.Tensor, bias: Optional[torch.Tensor],
                 num_experts: int, topk: int = 8, n_group: int = 8, topk_group: int = 4,
                 routed_scaling_factor: float = 2.5, renormalize: bool = True,
                 scoring_func: str = "sigmoid", swiglu_limit: float = 0.0, group=None,
                 steps=DeviceSteps, domain: Optional[PeerDomain] = None,
                 combine: str = "auto", push_chunks: int = 2):
        if domain is not None:
            group = domain.group
        group = as_exchange(group)
        world = group.world_size
        if num_experts % world:
            raise ValueError(f"num_experts={num_experts} is not a multiple of world size {world}")
        if w_gu.shape[0] != num_experts // world or w_down.shape[0] != num_experts // world:
            raise ValueError("w_gu / w_down must hold num_experts / world_size local experts")
        self.w_gu, self.w_down, self.bias = w_gu, w_down, bias
        self.num_experts, self.local_experts = num_experts, num_experts // world
        self.topk, self.n_group, self.topk_group = topk, n_group, topk_group
        self.routed_scaling_factor, self.renormalize = routed_scaling_factor, renormalize
        self.scoring_func, self.swiglu_limit = scoring_func, swiglu_limit
        self.group, self.steps, self.domain = group, steps, domain
        if domain is not None and domain.world_size != world:
            raise ValueError("the peer domain and the process group disagree on the world size")
        if combine not in ("auto", "fused", "push"):
            raise ValueError("combine must be 'auto', 'fused' or 'push'")
        # Peer transport: "fused" stores each weighted slot from the down-GEMM
        # epilogue straight into its source rank; "push" lets the GEMM write
        # locally and a row-coalesced kernel stream the rows over NVLink.  The
        # epilogue's per-thread 64-byte stores to remote memory hold its
        # accumulator longer, which stalls the GEMM as more rows leave the GPU
        # (measured on B200: equal at 2 ranks, push 1.3x faster at 8), so
        # "auto" pushes.
        self.combine = "push" if combine == "auto" else combine
        # "push" computes the down projection in `push_chunks` groups of
        # experts and streams each group's rows while the next one computes.
        self.push_chunks = max(1, min(push_chunks, self.local_experts))

    def gate(self, logits: torch.Tensor):
        return self.steps.topk_gating(logits, self.bias, self.topk, self.n_group, self.topk_group,
                                      self.routed_scaling_factor, self.renormalize,
                                      self.scoring_func)

    def experts(self, d: Dispatch, mark=None):
        """Expert side: permute, gate/up + SwiGLU, down.  Returns (y, s2d)."""
        permuted, offsets, s2d = expert_permute(d, self.local_experts, self.steps)
        if mark:
            mark("ep_expert_permute")
        h = self.steps.grouped_gemm_swiglu(permuted, self.w_gu, offsets, self.swiglu_limit)
        if mark:
            mark("gate_up_swiglu_gemm")
        y = self.steps.grouped_gemm(h, self.w_down, offsets)
        if mark:
            mark("down_gemm")
        return y, s2d

    def forward(self, hidden: torch.Tensor, logits: torch.Tensor,
                mark: Optional[Callable[[str], None]] = None) -> torch.Tensor:
        w, idx = self.gate(logits)
        if mark:
            mark("gating")
        if self.domain is not None:
            return self._forward_peer(hidden, idx, w, mark)
        d = dispatch(hidden, idx, w, self.num_experts, self.group, self.steps, mark)
        y, s2d = self.experts(d, mark)
        return combine(d, y, s2d, self.group, self.steps, mark)

    def _forward_peer(self, hidden, idx, w, mark):
        pd = peer_dispatch(self.domain, hidden, idx, w, self.num_experts, self.steps, mark)
        permuted, offsets, s2d, _ = self.steps.expert_permute(pd.recv_rows, pd.recv_ids,
                                                              self.local_experts, pd.valid_slots)
        if mark:
            mark("ep_expert_permute")
        h = self.steps.grouped_gemm_swiglu(permuted, self.w_gu, offsets, self.swiglu_limit)
        if mark:
            mark("gate_up_swiglu_gemm")
        if self.combine == "push":
            return self._down_and_push(pd, h, offsets, s2d, mark)
        dst_rank, dst_row, dst_w = peer_combine_plan(pd, s2d, self.steps)
        _C.ep_down_gemm_combine(self.domain.handle, h, self.w_down, offsets, dst_rank, dst_row,
                                dst_w, pd.epoch)
        if mark:
            mark("down_gemm_combine")
        return peer_combine_finish(pd, self.steps, mark)

    def _down_and_push(self, pd, h, offsets, s2d, mark):
        """Down projection in groups of experts; each group's weighted rows
        go to their source ranks on a second stream while the next group
        computes, and the last group's rows go in token chunks.  The combine
        plan runs on the push stream beside the first GEMM."""
        dom = pd.domain
        main = torch.cuda.current_stream()
        comm = dom.push_stream()
        start = torch.cuda.Event()
        start.record(main)
        comm.wait_event(start)
        with torch.cuda.stream(comm):
            dst_rank, dst_row, dst_w, order, count = peer_combine_plan_chunked(pd, s2d, self.steps)
        y = torch.empty(h.shape[0], self.w_down.shape[1], dtype=h.dtype, device=h.device)
        El, C = self.local_experts, self.push_chunks
        bounds = [(c * El) // C for c in range(C + 1)]
        for c in range(C - 1):
            lo, hi = bounds[c], bounds[c + 1]
            _C.grouped_gemm_bf16_out(y, h, self.w_down[lo:hi], offsets[lo:hi + 1])
            ready = torch.cuda.Event()
            ready.record(main)
            comm.wait_event(ready)
            with torch.cuda.stream(comm):
                _C.ep_combine_push(dom.handle, y, dst_rank, dst_row, dst_w, pd.epoch,
                                   row_lo=offsets[lo:lo + 1], row_hi=offsets[hi:hi + 1],
                                   publish=False)
        # The last group's rows go in token chunks, each publishing its chunk
        # (the earlier groups' rows precede them on the same stream).
        lo, hi = bounds[C - 1], bounds[C]
        _C.grouped_gemm_bf16_out(y, h, self.w_down[lo:hi], offsets[lo:hi + 1])
        if mark:
            mark("down_gemm_push")

        def push_chunk(c):
            with torch.cuda.stream(comm):
                _C.ep_combine_push_chunk(dom.handle, y, dst_rank, dst_row, dst_w, order, count,
                                         c, pd.epoch, row_lo=offsets[lo:lo + 1],
                                         row_hi=offsets[hi:hi + 1])

        return peer_combine_chunked(pd, push_chunk, comm, self.steps, mark)

    __call__ = forward


def replicated_forward(hidden: torch.Tensor, logits: torch.Tensor, bias: Optional[torch.Tensor],
                       w_gu: torch.Tensor, w_down: torch.Tensor, num_experts: int,
                       topk: int = 8, n_group: int = 8, topk_group: int = 4,
                       routed_scaling_factor: float = 2.5, renormalize: bool = True,
                       scoring_func: str = "sigmoid", swiglu_limit: float = 0.0, group=None,
                       steps=DeviceSteps) -> torch.Tensor:
    """The reference consumer's expert-parallel contract
    (smxx/permute/moe_permute.h:67-99; tests/test_kernels.py:131-142,
    187-200): every rank holds the same tokens and the experts are sharded
    (rank r owns experts [r*E/G, (r+1)*E/G), `w_gu` / `w_down` hold those).
    Each rank computes the per-slot rows bf16(w * y) of its own experts, zero
    for the other slots; a bf16 SUM all-reduce of the [T, topk, H] rows
    leaves every slot with its one non-zero contribution, and the fixed-order
    slot reduce gives [T, H].  Exact: a sum of one value and zeros is that
    value, so every rank returns the one-GPU canonical result bit for bit.
    Moves T*topk*H*2 bytes per rank through the all-reduce where the
    dispatch/combine path (EPMoELayer) moves only the rows that change rank.
    """
    ex = as_exchange(group)
    G, r = ex.world_size, ex.rank
    if num_experts % G:
        raise ValueError(f"num_experts={num_experts} is not a multiple of world size {G}")
    El = num_experts // G
    T = hidden.shape[0]
    w, idx = steps.topk_gating(logits, bias, topk, n_group, topk_group, routed_scaling_factor,
                               renormalize, scoring_func)
    permuted, offsets, s2d, _ = steps.moe_permute(hidden, idx, num_experts)
    local = offsets[r * El:(r + 1) * El + 1]
    h = steps.grouped_gemm_swiglu(permuted, w_gu, local, swiglu_limit)
    y = steps.grouped_gemm(h, w_down, local)
    lo, hi = (int(v) for v in local[[0, -1]].tolist())
    y[:lo].zero_()
    y[hi:].zero_()
    perslot = steps.unpermute_perslot(y, w, s2d, T, topk)
    ex.all_reduce_sum(perslot)
    return steps.reduce_slots(perslot)
