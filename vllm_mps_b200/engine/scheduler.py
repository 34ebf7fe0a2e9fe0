"""FCFS request scheduler (same algorithm as the reference's engine/scheduler.py:86-226).

Per step: (1) resume preempted groups that fit, (2) admit waiting groups
while the batch and the token budget allow (reserving every prompt slot),
(3) keep each already-running group if one more slot fits, else preempt it
(swap out), (4) append one slot per continuing sequence.  Like the
reference, step (3) checks each group on its own, so step (4) can still run
out of blocks when several groups share the last free block; the
``MemoryError`` propagates exactly as the reference's does.

``preempt_watermark`` (new, default None = the reference's behaviour) keeps
``(1 - watermark)`` of the GPU blocks free: a group is admitted, resumed or
kept only if its blocks fit without dipping into that reserve.
"""

from __future__ import annotations

import logging
import math
from collections import deque
from dataclasses import dataclass, field

from vllm_mps_b200.config import MAX_BATCH_SIZE, MAX_TOKENS_PER_STEP
from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
from vllm_mps_b200.core.sequence import SequenceGroup, SequenceStatus

logger = logging.getLogger(__name__)


@dataclass
class SchedulerOutput:
    scheduled_groups: list[SequenceGroup] = field(default_factory=list)
    preempted_groups: list[SequenceGroup] = field(default_factory=list)
    num_batched_tokens: int = 0
    num_scheduled_seqs: int = 0


class Scheduler:
    """Coordinates admission, preemption and batching over a :class:`KVCacheManager`."""

    def __init__(self, kv_cache_manager: KVCacheManager, max_batch_size: int = MAX_BATCH_SIZE,
                 max_tokens_per_step: int = MAX_TOKENS_PER_STEP,
                 preempt_watermark: float | None = None) -> None:
        self.kv_cache_manager = kv_cache_manager
        self.max_batch_size = max_batch_size
        self.max_tokens_per_step = max_tokens_per_step
        self.preempt_watermark = preempt_watermark
        self._waiting: deque[SequenceGroup] = deque()
        self._running: list[SequenceGroup] = []
        self._preempted: list[SequenceGroup] = []

    def add_request(self, group: SequenceGroup) -> None:
        self._waiting.append(group)
        logger.info("Scheduler: queued group=%d, waiting=%d", group.group_id, len(self._waiting))

    def _fits(self, seq_id: int, num_tokens: int) -> bool:
        kv = self.kv_cache_manager
        if self.preempt_watermark is None:
            return kv.can_allocate(seq_id, num_tokens)
        # KVCacheManager.can_allocate's block arithmetic, minus the reserve.
        total = kv.gpu_allocator.total_blocks
        reserve = int(math.floor(total * (1.0 - self.preempt_watermark)))
        return kv.blocks_needed(seq_id, num_tokens) <= kv.get_num_free_gpu_blocks() - reserve

    def _free_beyond_reserve(self) -> int:
        """Free GPU blocks minus the watermark's reserve (the count _fits compares with)."""
        kv = self.kv_cache_manager
        free = kv.get_num_free_gpu_blocks()
        if self.preempt_watermark is None:
            return free
        total = kv.gpu_allocator.total_blocks
        return free - int(math.floor(total * (1.0 - self.preempt_watermark)))

    def schedule(self) -> SchedulerOutput:
        scheduled: list[SequenceGroup] = []
        preempted: list[SequenceGroup] = []
        n_seqs = 0
        n_tokens = 0

        # 1. resume preempted groups (engine/scheduler.py:98-125)
        resumed: list[SequenceGroup] = []
        for group in list(self._preempted):
            if n_seqs >= self.max_batch_size:
                break
            seqs = group.get_seqs(SequenceStatus.PREEMPTED)
            total = sum(s.get_total_len() for s in seqs)
            if not all(self._fits(s.seq_id, s.get_total_len()) for s in seqs):
                continue
            for s in seqs:
                self.kv_cache_manager.swap_in(s.seq_id)
                s.status = SequenceStatus.RUNNING
            self._preempted.remove(group)
            self._running.append(group)
            scheduled.append(group)
            n_seqs += len(seqs)
            n_tokens += total
            resumed.append(group)

        # 2. admit waiting groups FCFS (:127-161)
        admitted: list[SequenceGroup] = []
        while self._waiting:
            if n_seqs >= self.max_batch_size:
                break
            group = self._waiting[0]
            seqs = group.get_seqs(SequenceStatus.WAITING)
            total = sum(s.get_total_len() for s in seqs)
            if n_tokens + total > self.max_tokens_per_step:
                break
            if not all(self._fits(s.seq_id, s.get_total_len()) for s in seqs):
                break
            self._waiting.popleft()
            for s in seqs:
                self.kv_cache_manager.allocate(s.seq_id)
                self.kv_cache_manager.append_slots(s.seq_id, s.get_prompt_len())
                s.status = SequenceStatus.RUNNING
            self._running.append(group)
            scheduled.append(group)
            n_seqs += len(seqs)
            n_tokens += total
            admitted.append(group)

        # 3. keep or preempt the groups that were already running (:163-187).
        # Every check asks for one token against the same free-block count
        # (nothing is allocated until step 4), so when at least one block is
        # free beyond the reserve every group fits and the checks are skipped.
        picked = {id(g) for g in scheduled}
        all_fit = self._free_beyond_reserve() >= 1
        for group in [g for g in self._running if id(g) not in picked]:
            seqs = group.get_seqs(SequenceStatus.RUNNING)
            if all_fit or all(self._fits(s.seq_id, 1) for s in seqs):
                scheduled.append(group)
                n_seqs += len(seqs)
                n_tokens += sum(s.get_total_len() for s in seqs)
            else:
                for s in seqs:
                    self.kv_cache_manager.swap_out(s.seq_id)
                    s.status = SequenceStatus.PREEMPTED
                self._running.remove(group)
                self._preempted.append(group)
                preempted.append(group)

        # 4. one new slot per continuing sequence (:189-196)
        fresh = {id(g) for g in admitted} | {id(g) for g in resumed}
        for group in scheduled:
            if id(group) in fresh:
                continue
            for s in group.get_seqs(SequenceStatus.RUNNING):
                self.kv_cache_manager.append_slot(s.seq_id)

        return SchedulerOutput(scheduled_groups=scheduled, preempted_groups=preempted,
                               num_batched_tokens=n_tokens, num_scheduled_seqs=n_seqs)

    def mark_finished(self, seq_id: int) -> None:
        """Finish ``seq_id``; free the group's blocks once every member is done (:208-226)."""
        for group in self._running:
            for s in group.sequences:
                if s.seq_id == seq_id:
                    s.status = SequenceStatus.FINISHED
                    if group.is_finished():
                        for seq in group.sequences:
                            self.kv_cache_manager.free(seq.seq_id)
                        self._running.remove(group)
                        logger.info("Scheduler: group=%d finished, memory freed", group.group_id)
                    return

    def get_num_waiting(self) -> int:
        return len(self._waiting)

    def get_num_running(self) -> int:
        return len(self._running)

    def get_num_preempted(self) -> int:
        return len(self._preempted)

    def __repr__(self) -> str:
        return (f"Scheduler(waiting={len(self._waiting)}, running={len(self._running)}, "
                f"preempted={len(self._preempted)})")
