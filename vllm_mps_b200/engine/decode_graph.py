"""CUDA-graph capture of the engine's decode step.

The reference runs every decode step as an eager HuggingFace forward
(models/llama_adapter.py:137-207): per layer a dozen PyTorch ops plus its
attention, each one a Python call and a kernel launch, so at small batch a
step is bound by the host (config 0 on a B200: ~7.5 ms per step for 22 layers,
almost all of it launch overhead).  Here the step's GPU work -- embedding,
every decoder layer (RMSNorm, fused QKV GEMM, the fused decode-step kernel,
O projection, RMSNorm, gated MLP, residuals), final norm and LM head -- is
captured once per batch bucket as a CUDA graph and replayed.

The forward replayed is the decoder layer's own sequence of HF submodules
(``input_layernorm``, attention, residual, ``post_attention_layernorm``,
``mlp``, residual; transformers' LlamaDecoderLayer.forward), minus the model
level work a decode step does not use (masks and rotary tables: RoPE runs
inside the decode kernel), so the logits are those of the eager path.

Per step the host packs block tables, lengths, positions, slots and token ids
of the batch, padded to the bucket (padding rows have length 0 and no slot:
the kernel writes zeros for them and touches no slot), into one pinned
buffer; one H2D copy moves it into the bucket's static device buffer and the
graph is replayed.  Block tables are ``max_blocks`` wide; a step whose
tables are wider, or a batch above the largest bucket, runs eagerly.
"""

from __future__ import annotations

import logging
from types import SimpleNamespace

import numpy as np
import torch

logger = logging.getLogger(__name__)

BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)


class DecodeGraphRunner:
    """Captures and replays one decode step of a Llama-family model per batch bucket."""

    def __init__(self, adapter, kv_cache_manager, block_size: int, max_blocks: int) -> None:
        m = adapter.hf_model
        for attr in ("embed_tokens", "layers", "norm"):
            if not hasattr(m.model, attr):
                raise ValueError(f"decode graphs need a Llama-family model (no model.{attr})")
        self.adapter = adapter
        self.kv = kv_cache_manager
        self.block_size = block_size
        self.max_blocks = int(max_blocks)
        self.device = adapter.model_config.device
        self._graphs: dict[int, tuple] = {}
        self._pool = None

    @staticmethod
    def bucket(batch: int) -> int | None:
        for b in BUCKETS:
            if b >= batch:
                return b
        return None

    # ── one step of the model on the static buffers ──────────────────────────

    def _forward(self, st) -> None:
        m = self.adapter.hf_model
        meta = st.meta
        x = m.model.embed_tokens(st.tokens).unsqueeze(1)
        for layer in m.model.layers:
            r = x
            h = layer.input_layernorm(x)
            x = r + layer.self_attn._attend(h, meta)
            r = x
            h = layer.post_attention_layernorm(x)
            x = r + layer.mlp(h)
        x = m.model.norm(x)
        st.logits.copy_(m.lm_head(x[:, 0, :]))

    def _static(self, Bb: int):
        """Static buffers of a bucket: [tables Bb x W | lengths | positions | slots | tokens]."""
        W = self.max_blocks
        n = Bb * W + 4 * Bb
        dev = torch.zeros(n, dtype=torch.int32, device=self.device)
        host = torch.zeros(n, dtype=torch.int32).pin_memory()
        o = Bb * W
        meta = SimpleNamespace(bt_tensor=dev[:o].view(Bb, W), sl_tensor=dev[o:o + Bb],
                               pos_tensor=dev[o + Bb:o + 2 * Bb],
                               slot_mapping=dev[o + 2 * Bb:o + 3 * Bb])
        vocab = self.adapter.hf_model.lm_head.out_features
        logits = torch.empty((Bb, vocab), dtype=self.adapter.model_config.dtype,
                             device=self.device)
        return SimpleNamespace(Bb=Bb, W=W, dev=dev, host=host, meta=meta,
                               tokens=dev[o + 3 * Bb:], logits=logits)

    def _stage(self, st, token_ids, seq_ids, positions, seq_lens) -> None:
        """Pack the batch (padded to the bucket) into pinned memory; one H2D copy."""
        B, Bb, W = len(seq_ids), st.Bb, st.W
        h = st.host.numpy()
        h[:] = 0
        bt = h[:Bb * W].reshape(Bb, W)
        for i, sid in enumerate(seq_ids):
            t = self.kv.get_block_table(sid)
            bt[i, :len(t)] = t
        o = Bb * W
        pos = np.asarray(positions, dtype=np.int64)
        blk = bt[np.arange(B), pos // self.block_size].astype(np.int64)
        h[o:o + B] = seq_lens
        h[o + Bb:o + Bb + B] = pos
        h[o + 2 * Bb:o + 3 * Bb] = -1  # padding rows own no slot
        h[o + 2 * Bb:o + 2 * Bb + B] = blk * self.block_size + pos % self.block_size
        h[o + 3 * Bb:o + 3 * Bb + B] = token_ids
        st.dev.copy_(st.host, non_blocking=True)

    def _capture(self, Bb: int):
        st = self._static(Bb)
        # Warm-up outside the graph (sizes each layer's workspace), then capture.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side), torch.no_grad():
            self._stage(st, [], [], [], [])  # all rows empty: no slot, zero output
            self._forward(st)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._pool), torch.no_grad():
            self._forward(st)
        torch.cuda.synchronize(self.device)
        logger.info("DecodeGraphRunner: captured the decode step for batch bucket %d", Bb)
        return g, st

    # ── public ───────────────────────────────────────────────────────────────

    def can_run(self, seq_ids) -> bool:
        if self.bucket(len(seq_ids)) is None:
            return False
        return all(len(self.kv.get_block_table(s)) <= self.max_blocks for s in seq_ids)

    def run(self, token_ids, seq_ids, positions, seq_lens) -> torch.Tensor:
        """Logits ``(B, vocab)`` of one decode step (a view of the bucket's static buffer)."""
        B = len(seq_ids)
        Bb = self.bucket(B)
        if Bb not in self._graphs:
            self._graphs[Bb] = self._capture(Bb)
        g, st = self._graphs[Bb]
        self._stage(st, token_ids, seq_ids, positions, seq_lens)
        g.replay()
        return st.logits[:B]

    def capture_all(self, max_batch: int) -> list[int]:
        """Capture every bucket up to ``max_batch`` now (a serving engine's startup)."""
        done = []
        for b in BUCKETS:
            if b > max(1, max_batch) and done:
                break
            if b not in self._graphs:
                self._graphs[b] = self._capture(b)
            done.append(b)
            if b >= max_batch:
                break
        return done

    def release(self) -> None:
        self._graphs.clear()
