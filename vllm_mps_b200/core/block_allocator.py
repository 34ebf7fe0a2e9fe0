"""FIFO block allocator (same contract as the reference's core/block_allocator.py).

Blocks are handed out from the front of a FIFO free list and returned to its
back, so a freed id is reused only after every never-used id has been handed
out (block_allocator.py:85, :204).  Slot indices therefore match the
reference bit for bit for the same operation stream.
"""

from __future__ import annotations

import logging
from collections import deque
from enum import Enum

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock

logger = logging.getLogger(__name__)


class BlockAllocatorType(Enum):
    """Which pool an allocator manages."""

    GPU = "gpu"
    CPU = "cpu"


class BlockAllocator:
    """Fixed pool of :class:`PhysicalBlock` descriptors with a FIFO free list."""

    def __init__(self, allocator_type: BlockAllocatorType, total_blocks: int) -> None:
        self.allocator_type = allocator_type
        self.total_blocks = total_blocks
        self.block_size = BLOCK_SIZE
        self._all_blocks: dict[int, PhysicalBlock] = {
            i: PhysicalBlock(block_id=i) for i in range(total_blocks)}
        self._free_list: deque[int] = deque(range(total_blocks))
        logger.info("BlockAllocator [%s] initialised with %d blocks of size %d",
                    allocator_type.value, total_blocks, self.block_size)

    def allocate(self) -> PhysicalBlock:
        """Pop the oldest free block (ref_count 1); ``MemoryError`` when empty."""
        if not self._free_list:
            raise MemoryError(f"BlockAllocator [{self.allocator_type.value}]: "
                              f"out of memory. 0 free blocks remaining.")
        block = self._all_blocks[self._free_list.popleft()]
        block.increment_ref()
        return block

    def free(self, block: PhysicalBlock) -> None:
        """Drop one reference; at zero the block is reset and queued at the back."""
        block.decrement_ref()
        if block.is_free:
            block.reset()
            self._free_list.append(block.block_id)

    def fork(self, block: PhysicalBlock) -> PhysicalBlock:
        """Share ``block`` copy-on-write (one more reference, no new block)."""
        if block.block_id not in self._all_blocks:
            raise ValueError(f"BlockAllocator [{self.allocator_type.value}]: "
                             f"block {block.block_id} is not managed by this allocator.")
        block.increment_ref()
        return block

    def get_num_free_blocks(self) -> int:
        return len(self._free_list)

    def get_num_used_blocks(self) -> int:
        return self.total_blocks - len(self._free_list)

    def get_utilisation(self) -> float:
        return self.get_num_used_blocks() / self.total_blocks

    def get_all_free_block_ids(self) -> list[int]:
        return list(self._free_list)

    def __repr__(self) -> str:
        return (f"BlockAllocator(type={self.allocator_type.value}, total={self.total_blocks}, "
                f"free={self.get_num_free_blocks()}, used={self.get_num_used_blocks()}, "
                f"utilisation={self.get_utilisation():.1%})")
