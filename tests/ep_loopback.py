"""G expert-parallel ranks as threads of one process: an in-process exchange
with the interface of layerstormexpertkernels_b200.ep.ProcessGroupExchange.
On a GPU every thread launches on the same (default) stream, so a receive,
enqueued after the barrier, is ordered after every sender's kernels.  Test
infrastructure only."""
from __future__ import annotations

import threading

import torch


class LoopbackHub:
    def __init__(self, world_size: int, timeout: float = 120.0):
        self.world_size = world_size
        self.barrier = threading.Barrier(world_size, timeout=timeout)
        self.posted = [None] * world_size

    def endpoint(self, rank: int) -> "LoopbackExchange":
        return LoopbackExchange(self, rank)

    def run(self, fn):
        """Runs fn(rank, exchange) on world_size threads; returns the results
        in rank order and re-raises the first failure."""
        results, errors = [None] * self.world_size, []

        def body(r):
            try:
                results[r] = fn(r, self.endpoint(r))
            except BaseException as exc:  # noqa: BLE001 - reported below
                errors.append(exc)
                self.barrier.abort()

        threads = [threading.Thread(target=body, args=(r,)) for r in range(self.world_size)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return results


class LoopbackExchange:
    def __init__(self, hub: LoopbackHub, rank: int):
        self.hub, self.rank, self.world_size = hub, rank, hub.world_size

    def all_to_all(self, send: torch.Tensor, send_splits: list[int],
                   recv_splits: list[int]) -> torch.Tensor:
        hub = self.hub
        assert len(send_splits) == self.world_size and sum(send_splits) == send.shape[0]
        starts = [0]
        for n in send_splits:
            starts.append(starts[-1] + n)
        hub.posted[self.rank] = (send, starts)
        hub.barrier.wait()
        parts = []
        for src in range(self.world_size):
            t, st = hub.posted[src]
            parts.append(t[st[self.rank]:st[self.rank + 1]])
        recv = torch.cat(parts) if parts else send[:0]
        assert [p.shape[0] for p in parts] == list(recv_splits)
        hub.barrier.wait()  # every rank has taken its slices before the next post
        return recv

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        hub = self.hub
        hub.posted[self.rank] = (t, None)
        hub.barrier.wait()
        total = hub.posted[0][0].float()
        for src in range(1, self.world_size):
            total = total + hub.posted[src][0].float()
        hub.barrier.wait()  # every rank has read every contribution
        t.copy_(total.to(t.dtype))
        return t
