"""KV-cache manager: every sequence's page table over a GPU and a CPU block pool.

Contract (reference ``core/kv_cache_manager.py:21-298``): ``can_allocate``
(read-only lookahead), ``allocate``/``append_slot``/``free`` of a sequence's
table, ``fork`` (the child shares the parent's blocks by reference count),
``swap_out``/``swap_in`` (each block moves to the other pool, in table order,
keeping its fill), ``get_block_table`` and pool counts.  Unknown sequences
raise ``KeyError``, duplicates ``ValueError``; a full pool ``MemoryError``.
``tests/test_slot_traces.py`` replays the reference's own recorded op streams
and requires identical tables and free counts after every operation.

The reference moves only block metadata on a swap, so a preempted
sequence's K/V is lost.  That stays the default; a ``swap_space`` (any
object with ``copy_out(gpu_ids, cpu_ids)`` and ``copy_in(cpu_ids, gpu_ids)``,
e.g. :class:`vllm_mps_b200.memory.cuda_memory_pool.SwapSpace`) makes the
swap carry the data too, without changing which ids are chosen.
"""

from __future__ import annotations

import logging

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock
from vllm_mps_b200.core.block_allocator import BlockAllocator, BlockAllocatorType
from vllm_mps_b200.core.block_table import BlockTable

logger = logging.getLogger(__name__)


class KVCacheManager:
    """Page tables of all live sequences over a GPU pool and a CPU swap pool."""

    def __init__(self, num_gpu_blocks: int, num_cpu_blocks: int, swap_space=None) -> None:
        self.block_size = BLOCK_SIZE
        self.gpu_allocator = BlockAllocator(BlockAllocatorType.GPU, num_gpu_blocks)
        self.cpu_allocator = BlockAllocator(BlockAllocatorType.CPU, num_cpu_blocks)
        self._tables: dict[int, BlockTable] = {}
        self.swap_space = swap_space

    def _table(self, seq_id: int) -> BlockTable:
        t = self._tables.get(seq_id)
        if t is None:
            raise KeyError(f"no page table for sequence {seq_id}")
        return t

    # ── lookahead ────────────────────────────────────────────────────────────

    def free_slots_in_last_block(self, seq_id: int) -> int:
        """Slots a sequence can still fill without a new block (0 if it has no table)."""
        t = self._tables.get(seq_id)
        return t.last_block_room() if t is not None else 0

    def blocks_needed(self, seq_id: int, num_tokens: int) -> int:
        """New GPU blocks that ``num_tokens`` more tokens of ``seq_id`` would take."""
        extra = num_tokens - self.free_slots_in_last_block(seq_id)
        return -(-extra // self.block_size) if extra > 0 else 0

    def can_allocate(self, seq_id: int, num_tokens: int) -> bool:
        return self.blocks_needed(seq_id, num_tokens) <= self.gpu_allocator.get_num_free_blocks()

    # ── lifecycle ────────────────────────────────────────────────────────────

    def has_sequence(self, seq_id: int) -> bool:
        return seq_id in self._tables

    def allocate(self, seq_id: int) -> None:
        if seq_id in self._tables:
            raise ValueError(f"sequence {seq_id} already has a page table")
        self._tables[seq_id] = BlockTable(seq_id, self.gpu_allocator)

    def append_slot(self, seq_id: int) -> PhysicalBlock:
        return self._table(seq_id).append_slot()

    def append_slots(self, seq_id: int, n: int) -> None:
        """``n`` calls of :meth:`append_slot` (a prompt's slots) in one go."""
        self._table(seq_id).append_slots(n)

    def free(self, seq_id: int) -> None:
        self._table(seq_id).free_all()
        del self._tables[seq_id]

    def fork(self, parent_seq_id: int, child_seq_id: int) -> None:
        parent = self._table(parent_seq_id)
        if child_seq_id in self._tables:
            raise ValueError(f"sequence {child_seq_id} already has a page table")
        ids = parent.block_ids().copy()
        for bid in ids.tolist():
            parent.allocator.share(bid)
        child = BlockTable(child_seq_id, parent.allocator)
        child.adopt(ids, parent.num_tokens(), parent.allocator)
        self._tables[child_seq_id] = child

    # ── swap (GPU <-> CPU) ───────────────────────────────────────────────────

    def _move(self, seq_id: int, src: BlockAllocator, dst: BlockAllocator) -> list[tuple[int, int]]:
        """Give every block of ``seq_id`` a ``dst`` block with the same fill; free the ``src`` one."""
        t = self._table(seq_id)
        moved = []
        for bid in t.block_ids().tolist():
            nid = dst.take()
            dst.counters.fill[nid] += src.counters.fill[bid]
            src.release(bid)
            moved.append((bid, nid))
        t.adopt([n for _, n in moved], t.num_tokens(), dst)
        return moved

    def swap_out(self, seq_id: int) -> None:
        moved = self._move(seq_id, self.gpu_allocator, self.cpu_allocator)
        if self.swap_space is not None and moved:
            self.swap_space.copy_out([g for g, _ in moved], [c for _, c in moved])
        logger.debug("sequence %d: %d blocks moved to the CPU pool", seq_id, len(moved))

    def swap_in(self, seq_id: int) -> None:
        moved = self._move(seq_id, self.cpu_allocator, self.gpu_allocator)
        if self.swap_space is not None and moved:
            self.swap_space.copy_in([c for c, _ in moved], [g for _, g in moved])
        logger.debug("sequence %d: %d blocks moved back to the GPU pool", seq_id, len(moved))

    # ── introspection ────────────────────────────────────────────────────────

    def get_block_ids(self, seq_id: int):
        """The block table of ``seq_id`` as a read-only int32 array."""
        return self._table(seq_id).block_ids()

    def get_block_table(self, seq_id: int) -> list[int]:
        return self._table(seq_id).get_all_physical_block_ids()

    def num_tokens(self, seq_id: int) -> int:
        """Token slots held by ``seq_id``."""
        return self._table(seq_id).num_tokens()

    def get_num_free_gpu_blocks(self) -> int:
        return self.gpu_allocator.get_num_free_blocks()

    def get_num_free_cpu_blocks(self) -> int:
        return self.cpu_allocator.get_num_free_blocks()

    def get_gpu_utilisation(self) -> float:
        return self.gpu_allocator.get_utilisation()

    def get_cpu_utilisation(self) -> float:
        return self.cpu_allocator.get_utilisation()

    def get_all_seq_ids(self) -> list[int]:
        return list(self._tables)

    def __repr__(self) -> str:
        g, c = self.gpu_allocator, self.cpu_allocator
        return (f"<KV cache: {len(self._tables)} sequences, GPU {g.get_num_used_blocks()}/"
                f"{g.total_blocks} blocks used, CPU {c.get_num_used_blocks()}/{c.total_blocks}>")
