"""Device KV-cache pool in HBM (replaces the reference's memory/mps_memory_pool.py).

Layout is the reference's: ``(num_blocks, 2, block_size, n_kv_heads, head_dim)``,
dim 1 = K (0) / V (1), zero-initialised (mps_memory_pool.py:62-66); this is
the layout the sm_100a kernels read with TMA.  The method set and the
``IndexError`` bounds checks are the reference's (:82-268).  Two modes:

* ``num_layers=None`` -- one pool shared by every layer, as the reference
  engine builds it (engine/llm_engine.py:166-173): every layer writes the
  current token into the same slot, so history slots hold the last layer's
  K/V.  Needed for token-for-token parity with the reference.
* ``num_layers=L`` -- one pool per layer in one allocation
  ``(L, num_blocks, 2, block_size, n_kv, D)``; :meth:`layer` returns layer
  ``i``'s pool (the physically meaningful cache).

``gather_*``/``read_*``/``write_kv`` are the reference's host-side helpers
(torch indexing on the device); the decode hot path does not use them --
the kernels read and write pages in place.
"""

from __future__ import annotations

import logging
from typing import Sequence

import torch

logger = logging.getLogger(__name__)


class CUDAMemoryPool:
    """Fixed-size KV pool tensor on a CUDA device (CPU allowed for host-only use)."""

    def __init__(self, num_blocks: int, block_size: int, n_heads: int, d_k: int,
                 dtype: torch.dtype = torch.float16, device: torch.device | str | None = None,
                 num_layers: int | None = None) -> None:
        if device is None:
            device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_heads = n_heads
        self.d_k = d_k
        self.dtype = dtype
        self.device = torch.device(device)
        self.num_layers = num_layers
        shape = (num_blocks, 2, block_size, n_heads, d_k)
        if num_layers is None:
            self._all = torch.zeros(shape, dtype=dtype, device=self.device)
            self._pool = self._all
        else:
            self._all = torch.zeros((num_layers, *shape), dtype=dtype, device=self.device)
            self._pool = self._all[0]
        logger.info("CUDAMemoryPool: shape=%s, %.2f MB on %s", list(self._all.shape),
                    self.get_memory_mb(), self.device)

    @classmethod
    def from_free_memory(cls, block_size: int, n_heads: int, d_k: int, dtype: torch.dtype,
                         device: torch.device | str, num_layers: int | None = None,
                         fraction: float = 0.85, max_blocks: int | None = None) -> "CUDAMemoryPool":
        """Size the pool to ``fraction`` of the device's free HBM (B200: ~180 GB)."""
        device = torch.device(device)
        free, _ = torch.cuda.mem_get_info(device)
        per_block = 2 * block_size * n_heads * d_k * torch.tensor([], dtype=dtype).element_size()
        per_block *= num_layers or 1
        n = int(free * fraction) // per_block
        if max_blocks is not None:
            n = min(n, max_blocks)
        if n <= 0:
            raise MemoryError("CUDAMemoryPool: no free device memory for a pool")
        return cls(n, block_size, n_heads, d_k, dtype, device, num_layers)

    def layer(self, i: int) -> torch.Tensor:
        """Pool tensor layer ``i`` reads and writes (the shared pool in shared mode)."""
        if self.num_layers is None:
            return self._pool
        return self._all[i]

    # ── single-token access (mps_memory_pool.py:82-135) ──────────────────────

    def write_kv(self, block_id: int, token_pos: int, k: torch.Tensor, v: torch.Tensor,
                 layer: int = 0) -> None:
        self._validate_indices(block_id, token_pos)
        pool = self.layer(layer)
        pool[block_id, 0, token_pos] = k
        pool[block_id, 1, token_pos] = v

    def read_kv(self, block_id: int, token_pos: int, layer: int = 0):
        self._validate_indices(block_id, token_pos)
        pool = self.layer(layer)
        return pool[block_id, 0, token_pos], pool[block_id, 1, token_pos]

    def read_block_kv(self, block_id: int, layer: int = 0):
        self._check_block(block_id, "block_id")
        pool = self.layer(layer)
        return pool[block_id, 0], pool[block_id, 1]

    # ── gathers (mps_memory_pool.py:139-209) ──────────────────────────────────

    def gather_blocks(self, block_ids: Sequence[int], layer: int = 0):
        ids = torch.as_tensor(list(block_ids), dtype=torch.long, device=self.device)
        return self.gather_blocks_tensor(ids, layer)

    def gather_blocks_tensor(self, ids_tensor: torch.Tensor, layer: int = 0):
        pool = self.layer(layer)
        k = pool[ids_tensor, 0].reshape(-1, self.n_heads, self.d_k)
        v = pool[ids_tensor, 1].reshape(-1, self.n_heads, self.d_k)
        return k, v

    def gather_blocks_batched(self, block_tables: list[list[int]], seq_lens: list[int],
                              max_seq_len: int, layer: int = 0):
        """Zero-padded ``(B, max_seq_len, n_heads, d_k)`` gather (kernels.gather_kv)."""
        from vllm_mps_b200.kernels import gather_kv

        B = len(block_tables)
        max_blocks = max(1, max(len(bt) for bt in block_tables))
        bt = torch.zeros(B, max_blocks, dtype=torch.int32)
        for i, row in enumerate(block_tables):
            bt[i, :len(row)] = torch.as_tensor(row, dtype=torch.int32)
        sl = torch.as_tensor(seq_lens, dtype=torch.int32)
        return gather_kv(self.layer(layer), bt.to(self.device), sl.to(self.device), max_seq_len)

    def copy_block(self, src_block_id: int, dst_block_id: int) -> None:
        """Copy a block's K/V (every layer in per-layer mode) (:211-228)."""
        self._check_block(src_block_id, "src_block_id")
        self._check_block(dst_block_id, "dst_block_id")
        if self.num_layers is None:
            self._all[dst_block_id] = self._all[src_block_id]
        else:
            self._all[:, dst_block_id] = self._all[:, src_block_id]

    # ── introspection ────────────────────────────────────────────────────────

    def get_memory_mb(self) -> float:
        return self._all.numel() * self._all.element_size() / (1024 * 1024)

    def utilisation_snapshot(self) -> dict:
        return {"device": str(self.device), "shape": list(self._all.shape),
                "memory_mb": self.get_memory_mb(), "num_blocks": self.num_blocks,
                "block_size": self.block_size, "dtype": str(self.dtype),
                "num_layers": self.num_layers}

    def __repr__(self) -> str:
        return (f"CUDAMemoryPool(device={self.device}, shape={list(self._all.shape)}, "
                f"memory={self.get_memory_mb():.2f} MB)")

    def _check_block(self, bid: int, label: str) -> None:
        if bid < 0 or bid >= self.num_blocks:
            raise IndexError(f"CUDAMemoryPool: {label} {bid} out of range "
                             f"(num_blocks={self.num_blocks}).")

    def _validate_indices(self, block_id: int, token_pos: int) -> None:
        """``IndexError`` on a bad block id or slot, like mps_memory_pool.py:257-268."""
        self._check_block(block_id, "block_id")
        if token_pos < 0 or token_pos >= self.block_size:
            raise IndexError(f"CUDAMemoryPool: token_pos {token_pos} out of range "
                             f"(block_size={self.block_size}).")


class SwapSpace:
    """Pinned host copy of swapped-out blocks: the data half of preemption.

    The reference's swap moves block metadata only and loses the KV data
    (core/kv_cache_manager.py:188, :225) and its CPU pool is never wired in
    (memory/cpu_memory_pool.py).  Attached to a :class:`KVCacheManager`, this
    copies the blocks' K/V (all layers) device->host on swap-out and back on
    swap-in, with one batched copy per direction on the caller's stream.
    """

    def __init__(self, gpu_pool: CUDAMemoryPool, num_cpu_blocks: int) -> None:
        self.gpu_pool = gpu_pool
        shape = list(gpu_pool._all.shape)
        blk_dim = 0 if gpu_pool.num_layers is None else 1
        shape[blk_dim] = num_cpu_blocks
        self._blk_dim = blk_dim
        self.cpu = torch.zeros(shape, dtype=gpu_pool.dtype)
        if torch.cuda.is_available():
            self.cpu = self.cpu.pin_memory()

    def copy_out(self, gpu_ids: list[int], cpu_ids: list[int]) -> None:
        g = torch.as_tensor(gpu_ids, dtype=torch.long, device=self.gpu_pool.device)
        data = self.gpu_pool._all.index_select(self._blk_dim, g).to("cpu")
        self.cpu.index_copy_(self._blk_dim, torch.as_tensor(cpu_ids, dtype=torch.long), data)

    def copy_in(self, cpu_ids: list[int], gpu_ids: list[int]) -> None:
        data = self.cpu.index_select(self._blk_dim, torch.as_tensor(cpu_ids, dtype=torch.long))
        g = torch.as_tensor(gpu_ids, dtype=torch.long, device=self.gpu_pool.device)
        self.gpu_pool._all.index_copy_(self._blk_dim, g, data.to(self.gpu_pool.device, non_blocking=True))
