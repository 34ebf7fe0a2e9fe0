"""Sequence-sharded serving across the GPUs of one node.

Decode and prefill have no dependency between sequences, so the engine
shards requests, not tensors: every rank (one process per GPU, launched by
torchrun) runs its own :class:`~vllm_mps_b200.engine.llm_engine.LLMEngine`
with a full weight replica, its own KV pool and its own block allocator (the
reference's single-device engine, engine/llm_engine.py:146-205, replicated).
Block ids are rank-local, so each rank's slotting is exactly the reference's
for the requests it owns.

The only collective is one ``all_gather_into_tensor`` per ``gather_every``
steps of a small int32 record per rank -- (global request id, sampled token,
finished) for every sequence that produced a token, plus a "work left" flag
-- used to assemble outputs on every rank and to end the loop on all ranks
at the same step.  Over NCCL the record is a device tensor (NVLink/NVSwitch); over gloo
(CPU tests) a host tensor.  Every rank takes the same number of collective
steps, including ranks whose shard is already finished, so no rank waits on
a collective the others never enter.
"""

from __future__ import annotations

import heapq
import time
from dataclasses import dataclass, field

import numpy as np
import torch


def shard_requests(costs: list[int], world: int) -> list[int]:
    """Rank of every request: longest-first greedy balance of ``costs``.

    ``costs[i]`` is the work of request i (prompt length + max new tokens).
    Requests are taken in decreasing cost (ties: lower index first) and each
    goes to the least-loaded rank (ties: lower rank), which keeps the largest
    per-rank total within one request of the mean.  Deterministic, so every
    rank computes the same assignment without communicating.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + int(costs[i]), r))
    return owner


@dataclass
class ShardedOutput:
    """Tokens of one request as assembled from every rank's records."""

    request_id: int
    rank: int
    token_ids: list[int] = field(default_factory=list)
    finished: bool = False


class ShardedEngine:
    """Runs one engine per rank and gathers sampled tokens every ``gather_every`` steps.

    ``engine`` is this rank's engine (anything with ``add_request(prompt,
    params) -> local id``, ``step() -> outputs with .request_id, .token_ids,
    .finished``, ``is_finished()``).  The record of a rank holds ``1 + 3 *
    capacity`` int32.  By default ``capacity`` is the largest number of
    requests any rank owns (every rank computes the same value from the
    shared assignment), which bounds the sequences a step can produce: the
    reference's scheduler admits waiting requests before it counts the
    running ones, so one step may schedule more than ``max_batch_size``
    (engine/scheduler.py:127-187).  A smaller explicit ``capacity`` saves
    bandwidth and is checked before every collective.

    With ``gather_every`` = k > 1 each rank buffers the tokens of k local
    steps and the ranks meet once per k steps (a record then holds
    ``1 + 3 * capacity * k`` int32).  The ranks run in lockstep only at the
    gathers, so a step that is long on one rank (a chunked prefill) and short
    on another is no longer paid as the slower of the two every step.

    The gathers do not stop the local loop: gather g is issued without
    waiting (over NCCL on a side stream, so it waits for no engine work) and
    read back at gather g + 1, by which time it has normally completed.  A
    rank that is ahead runs its next k steps instead of idling while a slower
    rank catches up; only when the whole run is imbalanced does one rank wait.
    The price is that the end of the run is seen one gather late: every rank
    stops at the gather after the one that showed all ranks done.
    """

    def __init__(self, engine, capacity: int | None = None, group=None,
                 device: torch.device | None = None, gather_every: int = 1):
        import torch.distributed as dist

        self.engine = engine
        self.capacity = None if capacity is None else int(capacity)
        if self.capacity is not None and self.capacity < 1:
            raise ValueError("capacity must be >= 1")
        if int(gather_every) < 1:
            raise ValueError("gather_every must be >= 1")
        self.gather_every = int(gather_every)
        # (global request id, token, finished) rows of the local steps since
        # the last gather, one int32 array per step.
        self._pending: list[np.ndarray] = []
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        backend = dist.get_backend(group)
        if device is None:
            device = (torch.device("cuda", torch.cuda.current_device()) if backend == "nccl"
                      else torch.device("cpu"))
        self.device = device
        self._local_to_global: dict[int, int] = {}
        self.outputs: dict[int, ShardedOutput] = {}
        self.steps = 0
        self.gathers = 0
        # Host wall time in local engine steps and in the gathers (the
        # gather's time includes waiting for the slowest rank to arrive).
        self.step_seconds = 0.0
        self.gather_seconds = 0.0
        self._rec = 0
        self._send = self._recv = None
        self._issued = None  # the gather in flight: (work, recv buffer, host landing, event)
        self._turn = 0
        self._side = None

    def _size_records(self, owner: list[int]) -> None:
        if self.capacity is None:
            counts = [0] * self.world
            for r in owner:
                counts[r] += 1
            self.capacity = max(1, max(counts))
        self._rec = 1 + 3 * self.capacity * self.gather_every
        # Two sets of buffers: gather g fills one while gather g - 1 is read from the other.
        pin = self.device.type == "cuda"
        self._send = [torch.empty(self._rec, dtype=torch.int32, device=self.device)
                      for _ in range(2)]
        self._recv = [torch.empty(self.world * self._rec, dtype=torch.int32, device=self.device)
                      for _ in range(2)]
        self._send_host = [torch.empty(self._rec, dtype=torch.int32, pin_memory=pin)
                           for _ in range(2)]
        self._recv_host = [torch.empty(self.world * self._rec, dtype=torch.int32,
                                       pin_memory=pin) for _ in range(2)]
        if pin:
            self._side = torch.cuda.Stream(self.device)

    def add_requests(self, prompts: list, params: list) -> list[int]:
        """Shard ``prompts`` over the ranks; this rank queues its own share.

        Global request ids are the indices into ``prompts``; every rank calls
        this with the same lists.  Returns the owner rank of each request.
        """
        if len(prompts) != len(params):
            raise ValueError("prompts and params differ in length")
        if self._send is not None:
            raise RuntimeError("add_requests may be called once per ShardedEngine")
        costs = [len(p) + sp.max_tokens for p, sp in zip(prompts, params)]
        owner = shard_requests(costs, self.world)
        self._size_records(owner)
        for gid, (p, sp) in enumerate(zip(prompts, params)):
            self.outputs[gid] = ShardedOutput(request_id=gid, rank=owner[gid])
            if owner[gid] == self.rank:
                local = self.engine.add_request(p, sp)
                self._local_to_global[local] = gid
        return owner

    def step(self, force_gather: bool = False) -> bool:
        """One local engine step; every ``gather_every`` calls (or when forced:
        every rank must pass the same value) a token gather.  Returns False
        once the ranks have seen a gather show every rank done; a forced
        gather is also read back at once (nothing left in flight)."""
        if self._send is None:
            self._size_records([])
        t0 = time.perf_counter()
        produced = self.engine.step() if not self.engine.is_finished() else []
        t1 = time.perf_counter()
        self.step_seconds += t1 - t0
        if len(produced) > self.capacity:
            raise RuntimeError(f"rank {self.rank}: {len(produced)} sequences in one step "
                               f"exceed the record capacity {self.capacity}")
        if produced:
            g2l = self._local_to_global
            self._pending.append(np.array(
                [(g2l[o.request_id], o.token_ids[-1], o.finished) for o in produced],
                dtype=np.int32))
        self.steps += 1
        if not force_gather and self.steps % self.gather_every:
            return True
        earlier = self._issued
        self._issue()
        more = self._collect(earlier) if earlier is not None else True
        if force_gather or not more:
            more = self._collect(self._issued)
            self._issued = None
        self.gather_seconds += time.perf_counter() - t1
        return more

    def _issue(self) -> None:
        """Start a gather of this rank's record; it is read back by ``_collect``."""
        import torch.distributed as dist

        j = self._turn
        self._turn ^= 1
        # The record is built and read as numpy arrays: element-wise torch
        # indexing cost ~3 ms per step at 256 sequences per rank.
        rec = self._send_host[j].numpy()
        rec[:] = -1
        rec[0] = 0 if self.engine.is_finished() else 1
        if self._pending:
            rows = np.concatenate(self._pending)
            rec[1:1 + rows.size] = rows.reshape(-1)
        self._pending.clear()
        send, recv = self._send[j], self._recv[j]
        if self._side is None:  # host tensors (gloo)
            work = dist.all_gather_into_tensor(recv, self._send_host[j], group=self.group,
                                               async_op=True)
            self._issued = (work, recv, None, None)
            return
        with torch.cuda.stream(self._side):
            send.copy_(self._send_host[j], non_blocking=True)
            work = dist.all_gather_into_tensor(recv, send, group=self.group, async_op=True)
            work.wait()  # the side stream waits for the collective
            self._recv_host[j].copy_(recv, non_blocking=True)
            done = torch.cuda.Event()
            done.record()
        self._issued = (work, recv, self._recv_host[j], done)

    def _collect(self, issued) -> bool:
        """Wait for a gather issued earlier and apply its tokens; whether any rank had work."""
        work, recv, host, done = issued
        if done is None:
            work.wait()
            allrec = recv.view(self.world, self._rec).numpy()
        else:
            done.synchronize()
            allrec = host.view(self.world, self._rec).numpy()
        self.gathers += 1
        more = bool((allrec[:, 0] > 0).any())
        slots = (self._rec - 1) // 3
        for r in range(self.world):
            body = allrec[r, 1:1 + 3 * slots].reshape(slots, 3)
            neg = np.flatnonzero(body[:, 0] < 0)
            n_r = int(neg[0]) if neg.size else slots
            if n_r == 0:
                continue
            body = body[:n_r]
            # Group the rows by request, keeping step order within a request
            # (a stable sort), so the Python loop runs per request, not per token.
            order = np.argsort(body[:, 0], kind="stable")
            gids = body[order, 0]
            starts = np.flatnonzero(np.r_[True, gids[1:] != gids[:-1]])
            ends = np.r_[starts[1:], n_r]
            toks = body[order, 1].tolist()
            fins = body[order, 2]
            for a, b, gid in zip(starts.tolist(), ends.tolist(), gids[starts].tolist()):
                o = self.outputs[gid]
                if o.rank != r:
                    raise RuntimeError(f"request {gid} reported by rank {r}, owned by {o.rank}")
                o.token_ids.extend(toks[a:b])
                o.finished = bool(fins[b - 1])
        return more

    def run(self, max_steps: int | None = None) -> dict[int, ShardedOutput]:
        """Step until every rank's shard is finished (or ``max_steps``)."""
        while True:
            last = max_steps is not None and self.steps + 1 >= max_steps
            more = self.step(force_gather=last)
            if not more or last:
                return self.outputs
