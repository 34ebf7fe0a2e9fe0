"""Per-sequence page table (same contract as the reference's core/block_table.py)."""

from __future__ import annotations

import logging

import numpy as np

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock
from vllm_mps_b200.core.block_allocator import BlockAllocator

logger = logging.getLogger(__name__)


class BlockTable:
    """Maps one sequence's token positions to physical blocks, allocated lazily."""

    def __init__(self, seq_id: int, allocator: BlockAllocator) -> None:
        self.seq_id = seq_id
        self.block_size = BLOCK_SIZE
        self._allocator = allocator
        self._blocks: list[PhysicalBlock] = []
        self._num_tokens = 0
        # The block ids as an int32 array, kept current by append_slot so a
        # decode step can copy a table without walking its blocks in Python;
        # rebuilt after replace_blocks (swap, fork).
        self._ids = np.empty(16, np.int32)
        self._ids_valid = True

    def append_slot(self) -> PhysicalBlock:
        """Add one token slot, allocating a block when the last one is full (:45-64)."""
        if not self._blocks or self._blocks[-1].is_full:
            block = self._allocator.allocate()
            self._blocks.append(block)
            if self._ids_valid:
                n = len(self._blocks)
                if n > len(self._ids):
                    self._ids = np.concatenate([self._ids, np.empty(len(self._ids), np.int32)])
                self._ids[n - 1] = block.block_id
        last = self._blocks[-1]
        last.add_tokens(1)
        self._num_tokens += 1
        return last

    def free_all(self) -> None:
        n = len(self._blocks)
        for block in self._blocks:
            self._allocator.free(block)
        self._blocks.clear()
        self._ids_valid = True
        self._num_tokens = 0
        logger.info("BlockTable [seq=%d]: freed %d blocks", self.seq_id, n)

    def get_block(self, logical_idx: int) -> PhysicalBlock:
        if logical_idx < 0 or logical_idx >= len(self._blocks):
            raise IndexError(f"BlockTable [seq={self.seq_id}]: logical index {logical_idx} "
                             f"out of range (num_blocks={len(self._blocks)}).")
        return self._blocks[logical_idx]

    def get_all_physical_block_ids(self) -> list[int]:
        """Ordered physical block ids (what the attention kernel reads)."""
        return [b.block_id for b in self._blocks]

    def replace_blocks(self, blocks: list[PhysicalBlock]) -> None:
        """Point the table at another list of blocks (swap, fork)."""
        self._blocks = blocks
        self._ids_valid = False

    def block_ids(self) -> np.ndarray:
        """The ordered physical block ids as an int32 array (read-only view)."""
        n = len(self._blocks)
        if not self._ids_valid:
            self._ids = np.empty(max(16, n), np.int32)
            self._ids[:n] = [b.block_id for b in self._blocks]
            self._ids_valid = True
        view = self._ids[:n]
        view.flags.writeable = False
        return view

    def get_last_block(self) -> PhysicalBlock:
        if not self._blocks:
            raise IndexError(f"BlockTable [seq={self.seq_id}]: table is empty.")
        return self._blocks[-1]

    def num_blocks(self) -> int:
        return len(self._blocks)

    def num_tokens(self) -> int:
        return self._num_tokens

    def is_empty(self) -> bool:
        return not self._blocks

    def __repr__(self) -> str:
        return (f"BlockTable(seq_id={self.seq_id}, num_blocks={len(self._blocks)}, "
                f"num_tokens={self._num_tokens}, block_ids={self.get_all_physical_block_ids()})")
