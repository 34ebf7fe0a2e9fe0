"""Block allocator over a fixed pool: int32 counter arrays and a FIFO ring of free ids.

Contract (reference ``core/block_allocator.py:20-150``): ``allocate`` hands out
the free block that has waited longest (a fresh pool hands out 0, 1, 2, ...;
a freed id joins the back of the queue), with one reference; ``free`` drops a
reference and queues the block again when none is left; ``fork`` adds a
reference; ``MemoryError`` when nothing is free; counts and utilisation.
That FIFO order is what makes slot indices identical to the reference's for
the same operation stream.

Layout: the free ids sit in an int32 ring buffer of ``total_blocks`` entries
(``head`` = oldest, ``n_free`` live entries), reference counts and fill
counts in the :class:`BlockCounters` arrays, one entry per block id.  The
integer methods (``take``, ``take_many``, ``release``) are what the block
tables use; ``allocate``/``free``/``fork`` keep the reference's
block-object interface on top of them.
"""

from __future__ import annotations

import logging
from enum import Enum

import numpy as np

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import BlockCounters, PhysicalBlock

logger = logging.getLogger(__name__)


class BlockAllocatorType(Enum):
    """Which pool an allocator manages."""

    GPU = "gpu"
    CPU = "cpu"


class BlockAllocator:
    """``total_blocks`` block ids handed out in FIFO order."""

    def __init__(self, allocator_type: BlockAllocatorType, total_blocks: int) -> None:
        n = int(total_blocks)
        if n < 0:
            raise ValueError(f"a pool cannot have {n} blocks")
        self.allocator_type = allocator_type
        self.total_blocks = n
        self.block_size = BLOCK_SIZE
        self.counters = BlockCounters(n, BLOCK_SIZE)
        self._ring = np.arange(n, dtype=np.int32)
        self._head = 0
        self._n_free = n
        self._handles: dict[int, PhysicalBlock] = {}
        logger.debug("%s pool: %d blocks of %d slots", allocator_type.value, n, BLOCK_SIZE)

    # ── integer interface ────────────────────────────────────────────────────

    def _out_of_blocks(self) -> MemoryError:
        return MemoryError(f"{self.allocator_type.value} pool exhausted: all "
                           f"{self.total_blocks} blocks are in use")

    def take(self) -> int:
        """Pop the oldest free id and give it one reference."""
        if self._n_free == 0:
            raise self._out_of_blocks()
        bid = int(self._ring[self._head])
        self._head += 1
        if self._head == self.total_blocks:
            self._head = 0
        self._n_free -= 1
        self.counters.ref[bid] = 1
        return bid

    def take_many(self, k: int) -> np.ndarray:
        """The next ``k`` free ids in FIFO order (as ``k`` calls of :meth:`take`)."""
        if k > self._n_free:
            raise self._out_of_blocks()
        idx = (self._head + np.arange(k)) % max(self.total_blocks, 1)
        ids = self._ring[idx].copy()
        self._head = (self._head + k) % max(self.total_blocks, 1)
        self._n_free -= k
        self.counters.ref[ids] = 1
        return ids

    def release(self, bid: int) -> None:
        """Drop one reference of ``bid``; when none is left, empty it and queue it last."""
        ref = self.counters.ref
        if ref[bid] <= 0:
            raise ValueError(f"block {bid} of the {self.allocator_type.value} pool is already free")
        ref[bid] -= 1
        if ref[bid] == 0:
            self.counters.fill[bid] = 0
            self._ring[(self._head + self._n_free) % self.total_blocks] = bid
            self._n_free += 1

    def share(self, bid: int) -> None:
        """One more reference on a block in use (copy-on-write sharing)."""
        if not 0 <= bid < self.total_blocks:
            raise ValueError(f"block {bid} is outside the {self.allocator_type.value} pool "
                             f"(0..{self.total_blocks - 1})")
        self.counters.ref[bid] += 1

    def block(self, bid: int) -> PhysicalBlock:
        """The handle of block ``bid`` (one per id, created on first use)."""
        h = self._handles.get(bid)
        if h is None:
            h = PhysicalBlock(bid, counters=self.counters, index=bid)
            self._handles[bid] = h
        return h

    # ── block-object interface ───────────────────────────────────────────────

    def allocate(self) -> PhysicalBlock:
        return self.block(self.take())

    def free(self, block: PhysicalBlock) -> None:
        if block._ctr is not self.counters:
            raise ValueError(f"block {block.block_id} does not belong to the "
                             f"{self.allocator_type.value} pool")
        self.release(block.block_id)

    def fork(self, block: PhysicalBlock) -> PhysicalBlock:
        self.share(block.block_id)
        return self.block(block.block_id)

    # ── counts ───────────────────────────────────────────────────────────────

    def get_num_free_blocks(self) -> int:
        return self._n_free

    def get_num_used_blocks(self) -> int:
        return self.total_blocks - self._n_free

    def get_utilisation(self) -> float:
        return self.get_num_used_blocks() / self.total_blocks if self.total_blocks else 0.0

    def get_all_free_block_ids(self) -> list[int]:
        """Free ids, the next to be handed out first."""
        if not self._n_free:
            return []
        idx = (self._head + np.arange(self._n_free)) % self.total_blocks
        return self._ring[idx].tolist()

    def __repr__(self) -> str:
        return (f"<{self.allocator_type.value} allocator: {self.get_num_used_blocks()} of "
                f"{self.total_blocks} blocks used>")
