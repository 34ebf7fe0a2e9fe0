"""LlamaForCausalLM adapter: injects PagedAttentionLayers (reference models/llama_adapter.py).

The injection hook is the reference's (:92-102): every ``layer.self_attn`` of
the HF model is replaced by ``PagedAttentionLayer.from_llama_layer(...)``,
and per-step metadata reaches the layers through the thread-local
``_batch_context`` (:26-34) rather than through HF's forward signature.

The metadata is built once per step for all layers, vectorised: block
tables, sequence lengths, positions and slot indices are assembled in
pinned host memory and copied to the device with one asynchronous copy each
(the reference fills the block table row by row and writes ``write_info``
with 2B scalar device writes, :175-196).  ``write_info`` is still provided
for callers of the reference's Metal-kernel interface.
"""

from __future__ import annotations

import logging
import threading
from types import SimpleNamespace

import numpy as np
import torch

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.layers.paged_attention_layer import PagedAttentionLayer
from vllm_mps_b200.models.base_adapter import BaseModelAdapter

logger = logging.getLogger(__name__)

_batch_context = threading.local()
_batch_context.is_batch = False
_batch_context.seq_ids = []
_batch_context.positions = []
_batch_context.seq_lens = []
_batch_context.bt_tensor = None      # int32 (B, max_blocks), zero-padded
_batch_context.write_info = None     # int32 (B, 2): (block_id, token_pos)
_batch_context.sl_tensor = None      # int32 (B,)
_batch_context.pos_tensor = None     # int32 (B,)
_batch_context.slot_mapping = None   # int32 (B,): block_id * block_size + token_pos
_batch_context.prefill = False       # rows are prompt tokens (engine prefill)
_batch_context.prefill_meta = None   # build_prefill_metadata(...) of the prefill chunk


def build_step_metadata(kv_cache_manager, seq_ids, positions, seq_lens, block_size: int,
                        device: torch.device) -> SimpleNamespace:
    """Device metadata of one decode step (one pinned host buffer, one copy).

    ``slot_mapping[i] = table_i[pos_i // block_size] * block_size + pos_i % block_size``,
    the reference's write target (layers/paged_attention_layer.py:318-324).
    """
    B = len(seq_ids)
    tables = [kv_cache_manager.get_block_table(s) for s in seq_ids]
    max_blocks = max(1, max(len(t) for t in tables))
    host = np.zeros((B, max_blocks + 3), dtype=np.int32)
    for i, t in enumerate(tables):
        host[i, :len(t)] = t
    pos = np.asarray(positions, dtype=np.int64)
    rows = np.arange(B)
    blk = host[rows, pos // block_size]
    host[:, max_blocks] = np.asarray(seq_lens, dtype=np.int32)
    host[:, max_blocks + 1] = pos
    host[:, max_blocks + 2] = blk * block_size + pos % block_size
    pinned = torch.from_numpy(host)
    if device.type == "cuda":
        pinned = pinned.pin_memory()
    dev = pinned.to(device, non_blocking=True)
    meta = SimpleNamespace(
        bt_tensor=dev[:, :max_blocks].contiguous(),
        sl_tensor=dev[:, max_blocks].contiguous(),
        pos_tensor=dev[:, max_blocks + 1].contiguous(),
        slot_mapping=dev[:, max_blocks + 2].contiguous(),
    )
    meta.write_info = torch.stack([meta.slot_mapping // block_size, meta.slot_mapping % block_size], 1)
    return meta


def build_prefill_metadata(kv_cache_manager, pieces, block_size: int,
                           device: torch.device) -> SimpleNamespace:
    """Device metadata of one prefill chunk (one pinned host buffer, one copy).

    ``pieces``: ``(seq_id, q_start, q_len)`` per sequence; the chunk's rows
    are the ``q_len`` tokens at positions ``q_start ..`` of each sequence in
    order.  Per row: position and slot (kernel 1 writes each row's K/V); per
    sequence: block table, ``q_start``, ``q_len`` and first row ``cu_q``
    (kernel 3 attends each row to its sequence's slots ``0..position``).
    """
    S = len(pieces)
    tables = [kv_cache_manager.get_block_table(sid) for sid, _, _ in pieces]
    max_blocks = max(1, max(len(t) for t in tables))
    q_start = np.array([qs for _, qs, _ in pieces], dtype=np.int64)
    q_lens = np.array([ql for _, _, ql in pieces], dtype=np.int64)
    rows = int(q_lens.sum())
    cu = np.zeros(S, dtype=np.int64)
    cu[1:] = np.cumsum(q_lens)[:-1]
    bt = np.zeros((S, max_blocks), dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    seq_of_row = np.repeat(np.arange(S), q_lens)
    pos = (np.arange(rows) - cu[seq_of_row] + q_start[seq_of_row]).astype(np.int64)
    slots = bt[seq_of_row, pos // block_size].astype(np.int64) * block_size + pos % block_size
    flat = np.concatenate([bt.reshape(-1), q_start, q_lens, cu, pos, slots]).astype(np.int32)
    pinned = torch.from_numpy(flat)
    if device.type == "cuda":
        pinned = pinned.pin_memory()
    dev = pinned.to(device, non_blocking=True)
    o = S * max_blocks
    return SimpleNamespace(
        bt_tensor=dev[:o].view(S, max_blocks), q_start=dev[o:o + S], q_lens=dev[o + S:o + 2 * S],
        cu_q=dev[o + 2 * S:o + 3 * S], pos_tensor=dev[o + 3 * S:o + 3 * S + rows],
        slot_mapping=dev[o + 3 * S + rows:o + 3 * S + 2 * rows],
        max_q_len=int(q_lens.max()) if S else 0, rows=rows)


class LlamaAdapter(BaseModelAdapter):
    """Adapter for LlamaForCausalLM and compatible architectures."""

    def __init__(self, model_name: str) -> None:
        self._model_name = model_name
        self.model_config = None
        self.hf_model = None
        self.tokenizer = None
        self.paged_layers: list[PagedAttentionLayer] = []
        self.kv_cache_manager = None
        self.memory_pool = None

    @property
    def model_name(self) -> str:
        return self._model_name

    def get_tokenizer(self):
        return self.tokenizer

    def load(self, model_config, kv_cache_manager, memory_pool) -> None:
        """Load weights from the HF hub / a local directory and inject (:58-108)."""
        from transformers import AutoModelForCausalLM, AutoTokenizer

        self.tokenizer = AutoTokenizer.from_pretrained(self._model_name)
        hf_model = AutoModelForCausalLM.from_pretrained(self._model_name,
                                                        torch_dtype=model_config.dtype)
        self.attach(hf_model, model_config, kv_cache_manager, memory_pool)

    def attach(self, hf_model, model_config, kv_cache_manager, memory_pool, tokenizer=None) -> None:
        """Inject PagedAttentionLayers into an already-built HF model (the :92-102 loop)."""
        self.model_config = model_config
        self.kv_cache_manager = kv_cache_manager
        self.memory_pool = memory_pool
        if tokenizer is not None:
            self.tokenizer = tokenizer
        self.hf_model = hf_model.to(device=model_config.device, dtype=model_config.dtype).eval()
        self.paged_layers = []
        for i, layer in enumerate(self.hf_model.model.layers):
            pl = PagedAttentionLayer.from_llama_layer(layer.self_attn, i, model_config,
                                                      kv_cache_manager, memory_pool)
            layer.self_attn = pl
            self.paged_layers.append(pl)
        logger.info("LlamaAdapter: injected %d PagedAttentionLayers", len(self.paged_layers))

    def forward_single_token(self, token_id: int, position_id: int, seq_id: int) -> torch.Tensor:
        """Logits ``(vocab,)`` of one token at ``position_id`` (:112-133)."""
        for pl in self.paged_layers:
            pl.set_context(seq_id, position_id)
        ids = torch.tensor([[token_id]], device=self.model_config.device, dtype=torch.long)
        with torch.no_grad():
            out = self.hf_model(input_ids=ids, use_cache=False)
        return out.logits[0, 0, :]

    def forward_batch(self, token_ids: list[int], seq_ids: list[int], positions: list[int],
                      seq_lens: list[int]) -> torch.Tensor:
        """Logits ``(B, vocab)`` of one decode step for B sequences (:137-207)."""
        device = self.model_config.device
        tok = torch.tensor(token_ids, dtype=torch.long)
        if device.type == "cuda":
            tok = tok.pin_memory()
        tok = tok.to(device, non_blocking=True)
        embeds = self.hf_model.model.embed_tokens(tok).unsqueeze(1)
        meta = build_step_metadata(self.kv_cache_manager, seq_ids, positions, seq_lens,
                                   BLOCK_SIZE, device)
        ctx = _batch_context
        ctx.is_batch = True
        ctx.seq_ids, ctx.positions, ctx.seq_lens = seq_ids, positions, seq_lens
        ctx.bt_tensor, ctx.sl_tensor = meta.bt_tensor, meta.sl_tensor
        ctx.pos_tensor, ctx.slot_mapping, ctx.write_info = meta.pos_tensor, meta.slot_mapping, meta.write_info
        try:
            with torch.no_grad():
                out = self.hf_model(inputs_embeds=embeds, use_cache=False)
        finally:
            ctx.is_batch = False
        return out.logits[:, 0, :]
