"""Drop-in replacement for HuggingFace ``LlamaAttention`` backed by the paged pool.

Same interface as the reference's layers/paged_attention_layer.py:26-391:
``from_llama_layer`` clones the q/k/v/o projections, ``forward(hidden_states,
**kwargs) -> (out, None)`` ignores HF's RoPE and mask and reads per-step
metadata from ``models.llama_adapter._batch_context``, ``set_context`` feeds
the single-token path, ``evict_sequence`` drops per-sequence caches.

The step between the projections -- RoPE on Q/K, the K/V write into the
sequence's slot, the paged gather, GQA and the softmax attention, which the
reference runs as per-sequence Python loops (:275-359) or as a Metal shader
-- is one call into the sm_100a kernel (``kernels.paged_decode_step``).  Q, K
and V come from one fused projection GEMM and are passed as strided slices
of its output, so nothing is copied or materialised.  There is no CPU path.
"""

from __future__ import annotations

import logging
import math

import torch
import torch.nn as nn

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
from vllm_mps_b200.core.model_config import ModelConfig
from vllm_mps_b200.layers.rotary_embedding import RotaryEmbedding

logger = logging.getLogger(__name__)


class PagedAttentionLayer(nn.Module):
    """Attention layer that writes and reads K/V through the paged pool."""

    def __init__(self, layer_idx: int, model_config: ModelConfig, kv_cache_manager: KVCacheManager,
                 memory_pool, W_Q: nn.Linear, W_K: nn.Linear, W_V: nn.Linear, W_O: nn.Linear,
                 rotary_emb: RotaryEmbedding) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.model_config = model_config
        self.kv_cache_manager = kv_cache_manager
        self.memory_pool = memory_pool
        self.W_Q, self.W_K, self.W_V, self.W_O = W_Q, W_K, W_V, W_O
        self.rotary_emb = rotary_emb
        self.n_heads = model_config.n_heads
        self.n_kv_heads = model_config.n_kv_heads
        self.d_k = model_config.d_k
        self.d_model = model_config.d_model
        self.block_size = BLOCK_SIZE
        self._current_seq_id: int | None = None
        self._current_position: int | None = None
        self.timer = None
        self._block_ids_cache: dict[int, tuple[tuple[int, ...], torch.Tensor]] = {}
        # One GEMM for Q, K and V: rows [W_Q; W_K; W_V].
        self.register_buffer("_w_qkv", torch.cat([W_Q.weight, W_K.weight, W_V.weight], 0).detach(),
                             persistent=False)
        self._workspace = None

    @classmethod
    def from_llama_layer(cls, layer, layer_idx: int, model_config: ModelConfig,
                         kv_cache_manager: KVCacheManager, memory_pool) -> "PagedAttentionLayer":
        """Build from a HuggingFace ``LlamaAttention``; weights are cloned (:91-148)."""
        dev, dt = model_config.device, model_config.dtype
        n_q, n_kv, D, d = model_config.n_heads, model_config.n_kv_heads, model_config.d_k, model_config.d_model

        def lin(src, out_f, in_f):
            m = nn.Linear(in_f, out_f, bias=False, device=dev, dtype=dt)
            m.weight.data.copy_(src.weight.data.to(device=dev, dtype=dt))
            return m

        if isinstance(layer, PagedAttentionLayer):  # a model already attached to an engine
            srcs = (layer.W_Q, layer.W_K, layer.W_V, layer.W_O)
        else:
            srcs = (layer.q_proj, layer.k_proj, layer.v_proj, layer.o_proj)
        W_Q = lin(srcs[0], n_q * D, d)
        W_K = lin(srcs[1], n_kv * D, d)
        W_V = lin(srcs[2], n_kv * D, d)
        W_O = lin(srcs[3], d, n_q * D)
        rot = RotaryEmbedding(D, model_config.max_seq_len, model_config.rope_theta, dev)
        return cls(layer_idx, model_config, kv_cache_manager, memory_pool, W_Q, W_K, W_V, W_O, rot)

    # ── forward ─────────────────────────────────────────────────────────────

    def forward(self, hidden_states: torch.Tensor, **kwargs):
        from vllm_mps_b200.models.llama_adapter import _batch_context

        if getattr(_batch_context, "is_batch", False):
            return self._forward_batch(hidden_states, _batch_context.seq_ids,
                                       _batch_context.positions, _batch_context.seq_lens)
        return self._forward_single(hidden_states)

    def _pool(self) -> torch.Tensor:
        return self.memory_pool.layer(self.layer_idx)

    def _workspace_buf(self):
        if self._workspace is None:
            from vllm_mps_b200.kernels import DecodeWorkspace

            self._workspace = DecodeWorkspace()
        return self._workspace

    @staticmethod
    def project(x2d: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``x2d @ w.T``: the decode GEMM kernel at decode batch sizes (M <= 8,
        weight streaming, chained to its neighbours with programmatic dependent
        launch), cuBLAS for everything else."""
        from vllm_mps_b200 import kernels as K

        if (x2d.is_cuda and x2d.stride(1) == 1 and x2d.stride(0) % 8 == 0
                and x2d.data_ptr() % 16 == 0 and w.is_contiguous() and w.data_ptr() % 16 == 0
                and K.decode_gemm_supported(x2d.shape[0], w.shape[0], w.shape[1])):
            return K.decode_gemm(x2d, w)
        return torch.matmul(x2d, w.t())

    def _attend(self, hidden_states: torch.Tensor, meta) -> torch.Tensor:
        """Fused QKV GEMM -> one decode-step kernel -> W_O, for (B, 1, d_model)."""
        from vllm_mps_b200.kernels import paged_decode_step

        B = hidden_states.shape[0]
        n_q, n_kv, D = self.n_heads, self.n_kv_heads, self.d_k
        qkv = self.project(hidden_states.reshape(B, self.d_model), self._w_qkv)
        q = qkv[:, : n_q * D].view(B, n_q, D)
        k = qkv[:, n_q * D: (n_q + n_kv) * D]
        v = qkv[:, (n_q + n_kv) * D:]
        out = paged_decode_step(q, k, v, meta.pos_tensor, meta.slot_mapping,
                                self.rotary_emb.inv_freq, self._pool(), meta.bt_tensor,
                                meta.sl_tensor, scale=1.0 / math.sqrt(D),
                                workspace=self._workspace_buf())
        if self.W_O.bias is None:
            return self.project(out.view(B, n_q * D), self.W_O.weight).view(B, 1, -1)
        return self.W_O(out.view(B, 1, n_q * D))

    def _prefill_rows(self, hidden_states: torch.Tensor, meta) -> torch.Tensor:
        """Prompt rows of a prefill chunk: kernel 1 writes every row's K/V, kernel 3 attends.

        Kernel 1 rotates q in place inside the fused QKV output and writes the
        rotated K and V of all rows into their slots; kernel 3 (tcgen05 causal
        prefill) then computes every row against its sequence's slots
        ``0..position`` -- the result of the reference's token-by-token
        single-token path (:175-241) for the whole chunk at once.

        ``hidden_states`` may carry padding rows after the chunk's
        ``meta.rows`` rows (a caller that rounds the GEMMs' row count): the
        projections run on every row, kernels 1 and 3 on the chunk's rows
        only, and the padding rows of the result are not meaningful.
        """
        from vllm_mps_b200.kernels import paged_prefill_attention, rope_reshape_and_cache

        B = hidden_states.shape[0]
        R = meta.rows
        n_q, n_kv, D = self.n_heads, self.n_kv_heads, self.d_k
        qkv = torch.matmul(hidden_states.reshape(B, self.d_model), self._w_qkv.t())
        q = qkv[:R, : n_q * D]
        k = qkv[:R, n_q * D: (n_q + n_kv) * D]
        v = qkv[:R, (n_q + n_kv) * D:]
        rope_reshape_and_cache(q, k, v, meta.pos_tensor, meta.slot_mapping,
                               self.rotary_emb.inv_freq, self._pool())
        out = torch.empty((B, n_q * D), dtype=qkv.dtype, device=qkv.device)
        if B > R:
            out[R:].zero_()
        paged_prefill_attention(q.view(R, n_q, D), self._pool(), meta.bt_tensor, meta.q_start,
                                meta.q_lens, meta.cu_q, meta.max_q_len, scale=1.0 / math.sqrt(D),
                                out=out[:R].view(R, n_q, D))
        return self.W_O(out.view(B, 1, n_q * D))

    def _write_kv_rows(self, hidden_states: torch.Tensor, meta) -> None:
        """Only the K/V half of :meth:`_prefill_rows`: the K and V projections
        and kernel 1's write of every row's rotated K and V (no query, no
        attention).  The last layer of a prefill needs nothing more: no later
        layer reads its output."""
        from vllm_mps_b200.kernels import rope_reshape_and_cache

        B, R = hidden_states.shape[0], meta.rows
        n_q, n_kv, D = self.n_heads, self.n_kv_heads, self.d_k
        kv = torch.matmul(hidden_states.reshape(B, self.d_model), self._w_qkv[n_q * D:].t())
        rope_reshape_and_cache(None, kv[:R, : n_kv * D], kv[:R, n_kv * D:], meta.pos_tensor,
                               meta.slot_mapping, self.rotary_emb.inv_freq, self._pool())

    def _forward_batch(self, hidden_states: torch.Tensor, seq_ids: list[int],
                       positions: list[int], seq_lens: list[int]):
        """Batched decode, one token per sequence (:245-364); prompt rows in prefill."""
        from vllm_mps_b200.models.llama_adapter import _batch_context

        if getattr(_batch_context, "prefill", False):
            return (self._prefill_rows(hidden_states, _batch_context.prefill_meta), None)
        return (self._attend(hidden_states, _batch_context), None)

    def _forward_single(self, hidden_states: torch.Tensor):
        """Single token at ``set_context``'s (seq_id, position) (:175-241)."""
        from vllm_mps_b200.models.llama_adapter import build_step_metadata

        seq_id, pos = self._current_seq_id, self._current_position
        if seq_id is None or pos is None:
            raise RuntimeError("PagedAttentionLayer: seq_id/position_id not set. "
                               "Call set_context() before forward.")
        meta = build_step_metadata(self.kv_cache_manager, [seq_id], [pos], [pos + 1],
                                   self.block_size, hidden_states.device)
        return (self._attend(hidden_states, meta), None)

    def set_context(self, seq_id: int, position_id: int) -> None:
        self._current_seq_id = seq_id
        self._current_position = position_id

    def _get_cached_ids_tensor(self, seq_id: int, block_ids: list[int]) -> torch.Tensor:
        """Per-sequence block-id tensor cache, rebuilt only when the table grows (:375-387)."""
        t = tuple(block_ids)
        cached = self._block_ids_cache.get(seq_id)
        if cached is None or cached[0] != t:
            tensor = torch.tensor(block_ids, dtype=torch.long, device=self.memory_pool.device)
            self._block_ids_cache[seq_id] = (t, tensor)
            return tensor
        return cached[1]

    def evict_sequence(self, seq_id: int) -> None:
        self._block_ids_cache.pop(seq_id, None)
