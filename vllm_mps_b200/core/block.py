"""One block of KV-cache memory, as a handle into its allocator's counter arrays.

Contract (reference ``core/block.py:15-99``): a block has an id, a reference
count, a count of filled token slots and a size; ``is_full``/``is_free``/
``num_empty_slots``; ``increment_ref``/``decrement_ref`` (``ValueError`` below
zero), ``add_tokens`` (``ValueError`` past the size) and ``reset``.

Layout here: an allocator keeps the counters of ALL its blocks in two int32
arrays (:class:`BlockCounters`), so a batch's bookkeeping can be read with
array indexing; a :class:`PhysicalBlock` is only (id, arrays, index).  A
block created on its own (``PhysicalBlock(7)``) gets private one-element
arrays and behaves the same.
"""

from __future__ import annotations

import numpy as np

from vllm_mps_b200.config import BLOCK_SIZE


class BlockCounters:
    """Reference counts and filled-slot counts of ``n`` blocks of ``block_size`` slots."""

    __slots__ = ("ref", "fill", "block_size")

    def __init__(self, n: int, block_size: int = BLOCK_SIZE) -> None:
        self.ref = np.zeros(n, np.int32)
        self.fill = np.zeros(n, np.int32)
        self.block_size = int(block_size)


class PhysicalBlock:
    """Handle on block ``block_id``; its counters live in a :class:`BlockCounters`."""

    __slots__ = ("block_id", "_ctr", "_at")

    def __init__(self, block_id: int, ref_count: int = 0, num_tokens: int = 0,
                 block_size: int = BLOCK_SIZE, *, counters: BlockCounters | None = None,
                 index: int | None = None) -> None:
        self.block_id = int(block_id)
        if counters is None:
            counters = BlockCounters(1, block_size)
            counters.ref[0] = ref_count
            counters.fill[0] = num_tokens
            index = 0
        self._ctr = counters
        self._at = int(block_id if index is None else index)

    # counters ---------------------------------------------------------------
    @property
    def ref_count(self) -> int:
        return int(self._ctr.ref[self._at])

    @ref_count.setter
    def ref_count(self, v: int) -> None:
        self._ctr.ref[self._at] = v

    @property
    def num_tokens(self) -> int:
        return int(self._ctr.fill[self._at])

    @num_tokens.setter
    def num_tokens(self, v: int) -> None:
        self._ctr.fill[self._at] = v

    @property
    def block_size(self) -> int:
        return self._ctr.block_size

    @property
    def is_full(self) -> bool:
        return int(self._ctr.fill[self._at]) == self._ctr.block_size

    @property
    def is_free(self) -> bool:
        return int(self._ctr.ref[self._at]) == 0

    @property
    def num_empty_slots(self) -> int:
        return self._ctr.block_size - int(self._ctr.fill[self._at])

    # updates ----------------------------------------------------------------
    def increment_ref(self) -> None:
        self._ctr.ref[self._at] += 1

    def decrement_ref(self) -> None:
        if self._ctr.ref[self._at] <= 0:
            raise ValueError(f"block {self.block_id} has no reference left to drop "
                             f"(ref_count {self.ref_count})")
        self._ctr.ref[self._at] -= 1

    def add_tokens(self, n: int) -> None:
        total = int(self._ctr.fill[self._at]) + n
        if total > self._ctr.block_size:
            raise ValueError(f"block {self.block_id} holds {self._ctr.block_size} slots; "
                             f"adding {n} to {self.num_tokens} filled would make {total}")
        self._ctr.fill[self._at] = total

    def reset(self) -> None:
        self._ctr.ref[self._at] = 0
        self._ctr.fill[self._at] = 0

    def __repr__(self) -> str:
        return (f"<block {self.block_id}: refs={self.ref_count} "
                f"filled={self.num_tokens}/{self.block_size}>")
