"""One sequence's page table: an int32 array of block ids, filled lazily.

Contract (reference ``core/block_table.py:19-130``): ``append_slot`` claims the
next token slot, taking a new block from the allocator only when the last
block is full; ``free_all`` returns every block (in table order); indexed and
last-block access raise ``IndexError`` out of range; counts of blocks and
tokens.

Layout: the ids live in a growable int32 array (``block_ids()`` returns a
read-only view of it, which is what a decode step copies into the device
block table) plus a token count; how full each block is lives in the
allocator's counter arrays, so blocks shared by a fork stay consistent.
"""

from __future__ import annotations

import numpy as np

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock
from vllm_mps_b200.core.block_allocator import BlockAllocator


class BlockTable:
    """Block ids of sequence ``seq_id`` in logical order."""

    def __init__(self, seq_id: int, allocator: BlockAllocator) -> None:
        self.seq_id = seq_id
        self.block_size = BLOCK_SIZE
        self.allocator = allocator
        self._ids = np.zeros(8, np.int32)
        self._n = 0
        self._tokens = 0

    def _grow_to(self, n: int) -> None:
        if n > len(self._ids):
            cap = max(n, 2 * len(self._ids))
            ids = np.zeros(cap, np.int32)
            ids[:self._n] = self._ids[:self._n]
            self._ids = ids

    def _last_has_room(self) -> bool:
        if self._n == 0:
            return False
        return int(self.allocator.counters.fill[self._ids[self._n - 1]]) < self.block_size

    # ── slots ────────────────────────────────────────────────────────────────

    def append_slot(self) -> PhysicalBlock:
        """Claim one token slot; returns the block that holds it."""
        a = self.allocator
        if not self._last_has_room():
            bid = a.take()
            self._grow_to(self._n + 1)
            self._ids[self._n] = bid
            self._n += 1
        last = int(self._ids[self._n - 1])
        a.counters.fill[last] += 1
        self._tokens += 1
        return a.block(last)

    def append_slots(self, n: int) -> None:
        """``n`` calls of :meth:`append_slot` at once (same blocks, same order)."""
        if n <= 0:
            return
        a, bs = self.allocator, self.block_size
        fill = a.counters.fill
        room = bs - int(fill[self._ids[self._n - 1]]) if self._n else 0
        first = min(room, n)
        new = -(-(n - first) // bs)
        if new > a.get_num_free_blocks():
            for _ in range(n):  # runs out part-way, exactly as single appends do
                self.append_slot()
            return
        if first:
            fill[self._ids[self._n - 1]] += first
        if new:
            ids = a.take_many(new)
            self._grow_to(self._n + new)
            self._ids[self._n:self._n + new] = ids
            self._n += new
            fill[ids] = bs
            fill[ids[-1]] = (n - first) - (new - 1) * bs
        self._tokens += n

    def free_all(self) -> None:
        """Return every block to the allocator, first block first."""
        for bid in self._ids[:self._n].tolist():
            self.allocator.release(bid)
        self._n = 0
        self._tokens = 0

    def adopt(self, ids, num_tokens: int, allocator: BlockAllocator) -> None:
        """Make the table hold ``ids`` of ``allocator`` with ``num_tokens`` tokens (fork, swap)."""
        ids = np.asarray(ids, np.int32)
        self.allocator = allocator
        self._n = 0
        self._grow_to(len(ids))
        self._ids[:len(ids)] = ids
        self._n = len(ids)
        self._tokens = int(num_tokens)

    # ── access ───────────────────────────────────────────────────────────────

    def get_block(self, logical_idx: int) -> PhysicalBlock:
        if not 0 <= logical_idx < self._n:
            raise IndexError(f"sequence {self.seq_id} has {self._n} blocks; "
                             f"no logical block {logical_idx}")
        return self.allocator.block(int(self._ids[logical_idx]))

    def get_last_block(self) -> PhysicalBlock:
        if self._n == 0:
            raise IndexError(f"sequence {self.seq_id} holds no block yet")
        return self.allocator.block(int(self._ids[self._n - 1]))

    def last_block_room(self) -> int:
        """Empty slots in the last block (0 for an empty table)."""
        if self._n == 0:
            return 0
        return self.block_size - int(self.allocator.counters.fill[self._ids[self._n - 1]])

    def get_all_physical_block_ids(self) -> list[int]:
        return self._ids[:self._n].tolist()

    def block_ids(self) -> np.ndarray:
        """The block ids as a read-only int32 view (valid until the table changes)."""
        view = self._ids[:self._n]
        view.flags.writeable = False
        return view

    def num_blocks(self) -> int:
        return self._n

    def num_tokens(self) -> int:
        return self._tokens

    def is_empty(self) -> bool:
        return self._n == 0

    def __repr__(self) -> str:
        return (f"<table of seq {self.seq_id}: {self._tokens} tokens in blocks "
                f"{self.get_all_physical_block_ids()}>")
