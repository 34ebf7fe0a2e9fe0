"""KV-cache manager: the single entry point for slot bookkeeping.

Same contract and the same slot assignment as the reference's
core/kv_cache_manager.py:21-298 (tests replay a recorded op stream of the
reference and require identical block tables after every operation).

Swap-out/in in the reference moves block *metadata* only; the KV data of a
preempted sequence is lost (kv_cache_manager.py:188, :225).  That stays the
default.  Attaching a ``swap_space`` (any object with ``copy_out(gpu_ids,
cpu_ids)`` and ``copy_in(cpu_ids, gpu_ids)``, e.g.
:class:`vllm_mps_b200.memory.cuda_memory_pool.SwapSpace`) makes swapping
carry the data too, without changing which block ids are chosen.
"""

from __future__ import annotations

import logging
import math

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock
from vllm_mps_b200.core.block_allocator import BlockAllocator, BlockAllocatorType
from vllm_mps_b200.core.block_table import BlockTable

logger = logging.getLogger(__name__)


class KVCacheManager:
    """Coordinates the GPU/CPU block allocators and the per-sequence tables."""

    def __init__(self, num_gpu_blocks: int, num_cpu_blocks: int, swap_space=None) -> None:
        self.block_size = BLOCK_SIZE
        self._gpu_allocator = BlockAllocator(BlockAllocatorType.GPU, num_gpu_blocks)
        self._cpu_allocator = BlockAllocator(BlockAllocatorType.CPU, num_cpu_blocks)
        self._block_tables: dict[int, BlockTable] = {}
        self.swap_space = swap_space
        logger.info("KVCacheManager: GPU=%d blocks, CPU=%d blocks, block_size=%d",
                    num_gpu_blocks, num_cpu_blocks, self.block_size)

    # ── lookahead ────────────────────────────────────────────────────────────

    def can_allocate(self, seq_id: int, num_tokens: int) -> bool:
        """Read-only check that ``num_tokens`` more slots fit (kv_cache_manager.py:53-77)."""
        if seq_id in self._block_tables:
            table = self._block_tables[seq_id]
            empty = table.get_last_block().num_empty_slots if not table.is_empty() else 0
            need_tokens = max(0, num_tokens - empty)
        else:
            need_tokens = num_tokens
        return math.ceil(need_tokens / self.block_size) <= self._gpu_allocator.get_num_free_blocks()

    # ── lifecycle ────────────────────────────────────────────────────────────

    def allocate(self, seq_id: int) -> None:
        if seq_id in self._block_tables:
            raise ValueError(f"KVCacheManager: seq_id {seq_id} already exists.")
        self._block_tables[seq_id] = BlockTable(seq_id, self._gpu_allocator)
        logger.info("KVCacheManager: allocated table for seq=%d", seq_id)

    def append_slot(self, seq_id: int) -> PhysicalBlock:
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        return self._block_tables[seq_id].append_slot()

    def free(self, seq_id: int) -> None:
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        self._block_tables[seq_id].free_all()
        del self._block_tables[seq_id]
        logger.info("KVCacheManager: freed table for seq=%d", seq_id)

    def fork(self, parent_seq_id: int, child_seq_id: int) -> None:
        """Child shares the parent's blocks copy-on-write (:134-172)."""
        if parent_seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: parent seq_id {parent_seq_id} not found.")
        if child_seq_id in self._block_tables:
            raise ValueError(f"KVCacheManager: child seq_id {child_seq_id} already exists.")
        parent = self._block_tables[parent_seq_id]
        child = BlockTable(child_seq_id, self._gpu_allocator)
        for block in parent._blocks:
            self._gpu_allocator.fork(block)
        child.replace_blocks(list(parent._blocks))
        child._num_tokens = parent._num_tokens
        self._block_tables[child_seq_id] = child
        logger.info("KVCacheManager: forked seq=%d -> seq=%d, %d blocks shared",
                    parent_seq_id, child_seq_id, len(parent._blocks))

    # ── swap (GPU <-> CPU) ───────────────────────────────────────────────────

    def swap_out(self, seq_id: int) -> None:
        """Move a sequence's blocks to the CPU pool (:176-211), data too if a swap space is set."""
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        table = self._block_tables[seq_id]
        new_blocks, pairs = [], []
        for gpu_block in table._blocks:
            cpu_block = self._cpu_allocator.allocate()
            cpu_block.add_tokens(gpu_block.num_tokens)
            pairs.append((gpu_block.block_id, cpu_block.block_id))
            self._gpu_allocator.free(gpu_block)
            new_blocks.append(cpu_block)
        if self.swap_space is not None and pairs:
            self.swap_space.copy_out([g for g, _ in pairs], [c for _, c in pairs])
        table.replace_blocks(new_blocks)
        table._allocator = self._cpu_allocator
        logger.info("KVCacheManager: swapped out seq=%d, %d blocks to CPU", seq_id, len(pairs))

    def swap_in(self, seq_id: int) -> None:
        """Move a sequence's blocks back to the GPU pool (:213-248)."""
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        table = self._block_tables[seq_id]
        new_blocks, pairs = [], []
        for cpu_block in table._blocks:
            gpu_block = self._gpu_allocator.allocate()
            gpu_block.add_tokens(cpu_block.num_tokens)
            pairs.append((cpu_block.block_id, gpu_block.block_id))
            self._cpu_allocator.free(cpu_block)
            new_blocks.append(gpu_block)
        if self.swap_space is not None and pairs:
            self.swap_space.copy_in([c for c, _ in pairs], [g for _, g in pairs])
        table.replace_blocks(new_blocks)
        table._allocator = self._gpu_allocator
        logger.info("KVCacheManager: swapped in seq=%d, %d blocks to GPU", seq_id, len(pairs))

    # ── introspection ────────────────────────────────────────────────────────

    def get_block_ids(self, seq_id: int):
        """``get_block_table`` as a read-only int32 numpy array (no per-call list)."""
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        return self._block_tables[seq_id].block_ids()

    def get_block_table(self, seq_id: int) -> list[int]:
        """Ordered physical block ids of ``seq_id`` (:252-265)."""
        if seq_id not in self._block_tables:
            raise KeyError(f"KVCacheManager: seq_id {seq_id} not found.")
        return self._block_tables[seq_id].get_all_physical_block_ids()

    def get_num_free_gpu_blocks(self) -> int:
        return self._gpu_allocator.get_num_free_blocks()

    def get_num_free_cpu_blocks(self) -> int:
        return self._cpu_allocator.get_num_free_blocks()

    def get_gpu_utilisation(self) -> float:
        return self._gpu_allocator.get_utilisation()

    def get_cpu_utilisation(self) -> float:
        return self._cpu_allocator.get_utilisation()

    def get_all_seq_ids(self) -> list[int]:
        return list(self._block_tables.keys())

    def __repr__(self) -> str:
        return (f"KVCacheManager(seqs={len(self._block_tables)}, "
                f"GPU free={self.get_num_free_gpu_blocks()}/{self._gpu_allocator.total_blocks}, "
                f"CPU free={self.get_num_free_cpu_blocks()}/{self._cpu_allocator.total_blocks}, "
                f"GPU util={self.get_gpu_utilisation():.1%}, CPU util={self.get_cpu_utilisation():.1%})")
