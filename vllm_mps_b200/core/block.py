"""Physical block descriptor: the unit of KV-cache memory (no tensors).

Same contract as the reference's core/block.py:15-99.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from vllm_mps_b200.config import BLOCK_SIZE


@dataclass
class PhysicalBlock:
    """Descriptor of one block of the pool.

    Attributes:
        block_id:   index into the pool's block dimension.
        ref_count:  sequences currently pointing at this block.
        num_tokens: filled token slots.
        block_size: token slots per block.
    """

    block_id: int
    ref_count: int = 0
    num_tokens: int = 0
    block_size: int = field(default=BLOCK_SIZE)

    @property
    def is_full(self) -> bool:
        return self.num_tokens == self.block_size

    @property
    def is_free(self) -> bool:
        return self.ref_count == 0

    @property
    def num_empty_slots(self) -> int:
        return self.block_size - self.num_tokens

    def increment_ref(self) -> None:
        self.ref_count += 1

    def decrement_ref(self) -> None:
        """Drop one reference; ``ValueError`` below zero (block.py:54-65)."""
        if self.ref_count <= 0:
            raise ValueError(
                f"Cannot decrement ref_count of block {self.block_id}: "
                f"ref_count is already {self.ref_count}.")
        self.ref_count -= 1

    def add_tokens(self, n: int) -> None:
        """Mark ``n`` more slots filled; ``ValueError`` past the block size (:67-82)."""
        if self.num_tokens + n > self.block_size:
            raise ValueError(
                f"Cannot add {n} tokens to block {self.block_id}: would have "
                f"{self.num_tokens + n} tokens but block_size is {self.block_size}.")
        self.num_tokens += n

    def reset(self) -> None:
        """Back to empty (used when the block returns to the free list)."""
        self.num_tokens = 0
        self.ref_count = 0

    def __repr__(self) -> str:
        return (f"PhysicalBlock(block_id={self.block_id}, ref_count={self.ref_count}, "
                f"num_tokens={self.num_tokens}, block_size={self.block_size})")
