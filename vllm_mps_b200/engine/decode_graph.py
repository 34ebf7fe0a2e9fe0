"""CUDA-graph capture of the engine's decode step.

The reference runs every decode step as an eager HuggingFace forward
(models/llama_adapter.py:137-207): per layer a dozen PyTorch ops plus its
attention, each one a Python call and a kernel launch, so at small batch a
step is bound by the host (config 0 on a B200: ~7.5 ms per step for 22 layers,
almost all of it launch overhead).  Here the step's GPU work -- embedding,
every decoder layer (RMSNorm, fused QKV GEMM, the fused decode-step kernel,
O projection, RMSNorm, gated MLP, residuals), final norm and LM head -- is
captured once per batch bucket as a CUDA graph and replayed.

For Llama-family layers (RMSNorm, bias-free SiLU-gated MLP) the replayed
forward is 8 kernels per layer: the QKV GEMM, the fused decode-step kernel,
the O GEMM, residual add + RMSNorm (``kernels.add_rmsnorm``), one [gate|up]
GEMM (the two weights are re-pointed as views into one buffer), SiLU * up
(``kernels.silu_mul``), the down GEMM, and residual add + the next RMSNorm.
At decode batch sizes (buckets up to 8) the GEMMs are the decode GEMM kernel
(``kernels.decode_gemm``: weight streaming, SiLU * up fused into the
[gate|up] GEMM, so 7 kernels per layer), all chained with programmatic
dependent launch; larger buckets use cuBLAS.  These are
the ops of transformers' LlamaDecoderLayer / LlamaRMSNorm / LlamaMLP with
their rounding points, minus the model-level work a decode step does not use
(masks and rotary tables: RoPE runs inside the decode kernel).  Other models
replay the HF submodules in the same order.

Per step the host packs block tables, lengths, positions, slots, token ids
and token sources of the batch, padded to the bucket (padding rows have
length 0 and no slot: the kernel writes zeros for them and touches no slot),
into one of the bucket's two pinned buffers (alternating, so packing step
k+1 never overwrites a buffer whose copy for step k may still be queued);
one H2D copy moves it into the bucket's static device buffer and the graph
is replayed.  The graph's first kernel (``kernels.embed_rmsnorm``) takes row
i's token from the host ids, or -- when its source entry is >= 0 -- from
``prev_tokens``, the device buffer the previous step's sampler wrote: that
is what lets a pipelined engine launch a step before it has read the last
one's tokens back.  Block tables are ``max_blocks`` wide; a step whose tables
are wider, or a batch above the largest bucket, runs eagerly.
"""

from __future__ import annotations

import logging
from types import SimpleNamespace

import numpy as np
import torch

logger = logging.getLogger(__name__)

BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)
# Prefill chunks run their GEMMs on a row count rounded up to this multiple:
# cuBLAS spends ~1 ms of host time choosing a kernel the first time it sees
# a shape (then ~20 us), so a serving run whose chunks all differ in length
# would pay that per chunk and GEMM; rounded, a run meets at most
# max_prefill_rows / 128 row counts, and ``warm_prefill_gemms`` can meet
# them all at startup.
PREFILL_ROW_ALIGN = 128


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
        self._gate_up = self._fuse_gate_up() if self._llama_layers() else None
        # Sampled ids of the last step, one per batch row (written by the
        # engine's sampler, read by the next replay through the source row).
        self.prev_tokens = torch.zeros(BUCKETS[-1], dtype=torch.long, device=self.device)

    def _llama_layers(self) -> bool:
        """Whether every layer is RMSNorm + bias-free SiLU-gated MLP (the fused path)."""
        import torch.nn as nn

        m = self.adapter.hf_model.model
        hid = self.adapter.model_config.d_model
        for layer in m.layers:
            mlp = getattr(layer, "mlp", None)
            for name in ("input_layernorm", "post_attention_layernorm"):
                if not hasattr(getattr(layer, name, None), "variance_epsilon"):
                    return False
            if mlp is None or not all(hasattr(mlp, a) for a in ("gate_proj", "up_proj", "down_proj")):
                return False
            act = getattr(mlp, "act_fn", None)
            # transformers' SiLU is its own module class (SiLUActivation).
            if not (isinstance(act, nn.SiLU) or type(act).__name__ == "SiLUActivation"):
                return False
            if any(getattr(mlp, a).bias is not None for a in ("gate_proj", "up_proj")):
                return False
            if mlp.gate_proj.out_features % 8 or hid % 8:
                return False
        # The embedding lookup is fused into the first kernel: a plain table.
        if type(m.embed_tokens) is not nn.Embedding or m.embed_tokens.max_norm is not None:
            return False
        return hasattr(m.norm, "variance_epsilon")

    def _fuse_gate_up(self) -> list[torch.Tensor]:
        """One [gate; up] weight per layer; the modules' weights become views of it."""
        import torch.nn as nn

        fused = []
        for layer in self.adapter.hf_model.model.layers:
            g, u = layer.mlp.gate_proj, layer.mlp.up_proj
            w = torch.cat([g.weight.detach(), u.weight.detach()], 0).contiguous()
            inter = g.out_features
            g.weight = nn.Parameter(w[:inter], requires_grad=False)
            u.weight = nn.Parameter(w[inter:], requires_grad=False)
            fused.append(w)
        return fused

    @property
    def fused(self) -> bool:
        """Whether the replayed step uses the fused element-wise kernels."""
        return self._gate_up is not None

    def own_kernels_per_step(self, batch: int) -> int:
        """How many of this library's kernels one replayed step of ``batch`` launches."""
        from vllm_mps_b200 import kernels as K

        m = self.adapter.hf_model
        nl = len(m.model.layers)
        if self._gate_up is None:
            return nl  # the decode-step kernel; the rest is HF modules
        Bb = self.bucket(batch) or batch
        d = self.adapter.model_config.d_model
        a0 = m.model.layers[0].self_attn
        # decode step; residual + RMSNorm twice a layer; embedding + the first RMSNorm
        n = nl + 2 * nl + 1
        n += nl * (K.decode_gemm_supported(Bb, a0._w_qkv.shape[0], d)
                   + K.decode_gemm_supported(Bb, d, a0.W_O.in_features))
        n += nl  # the [gate|up] decode GEMM with SiLU * up, or silu_mul after cuBLAS
        down = m.model.layers[0].mlp.down_proj
        n += nl * K.decode_gemm_supported(Bb, down.out_features, down.in_features)
        n += K.decode_gemm_supported(Bb, m.lm_head.out_features, d)
        return n

    @staticmethod
    def bucket(batch: int) -> int | None:
        for b in BUCKETS:
            if b >= batch:
                return b
        return None

    # ── one step of the model on the static buffers ──────────────────────────

    def _forward(self, st) -> None:
        if self._gate_up is not None:
            return self._forward_fused(st)
        m = self.adapter.hf_model
        meta = st.meta
        # Device-sourced tokens are a fused-path feature: ``run`` refuses them here.
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

    def _forward_fused(self, st) -> None:
        """Tokens, embedding and the first RMSNorm in one kernel; then per
        layer: QKV GEMM, decode-step kernel, O GEMM, add+RMSNorm, [gate|up]
        GEMM, SiLU*up, down GEMM, add+RMSNorm (the next layer's input norm, or
        the final norm) -- 8 kernels."""
        from vllm_mps_b200 import kernels as K
        from vllm_mps_b200.layers.paged_attention_layer import PagedAttentionLayer

        project = PagedAttentionLayer.project
        m = self.adapter.hf_model
        layers = m.model.layers
        first = layers[0].input_layernorm
        # res (Bb, d): the residual stream; h: its normalised copy.
        res, h = K.embed_rmsnorm(m.model.embed_tokens.weight, first.weight,
                                 first.variance_epsilon, st.tokens, src=st.src,
                                 prev=self.prev_tokens)
        Bb, d = res.shape
        for i, layer in enumerate(layers):
            attn = layer.self_attn._attend(h.unsqueeze(1), st.meta)
            post = layer.post_attention_layernorm
            K.add_rmsnorm(res, post.weight, post.variance_epsilon, delta=attn.view_as(res), out=h)
            gu = self._gate_up[i]
            if K.decode_gemm_supported(Bb, gu.shape[0] // 2, d, True):
                act = K.decode_gemm(h, gu, silu_mul=True)  # [gate|up] GEMM + SiLU * up
            else:
                act = K.silu_mul(torch.matmul(h, gu.t()))
            down = layer.mlp.down_proj
            mlp_out = project(act, down.weight) if down.bias is None else down(act)
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else m.model.norm
            K.add_rmsnorm(res, nxt.weight, nxt.variance_epsilon, delta=mlp_out, out=h)
        head = m.lm_head
        if head.bias is None and K.decode_gemm_supported(Bb, head.out_features, d):
            K.decode_gemm(h, head.weight, out=st.logits)
        else:
            st.logits.copy_(head(h))

    def prefill_rows(self, tokens: torch.Tensor, meta) -> None:
        """Write every layer's K/V for the prompt rows of one prefill chunk.

        The fused Llama layer sequence of the decode step, eager and at the
        chunk's row count: ``embed_rmsnorm``, then per layer kernel 1 + kernel
        3 (``PagedAttentionLayer._prefill_rows``), residual add + RMSNorm, the
        [gate | up] GEMM, SiLU * up, the down GEMM and residual add + the next
        RMSNorm; the last layer only projects and writes its K/V (nothing
        reads its attention or MLP output).  Unlike the HF forward it builds
        no causal mask (transformers' mask helpers read the device, a stall
        per chunk) and no rotary table.  ``tokens``: int32 on the device,
        the chunk's ``meta.rows`` ids followed by any padding (the GEMMs run
        on every row; ``padded_rows`` gives the engine's row count);
        ``meta``: ``build_prefill_metadata`` of the chunk.
        """
        from vllm_mps_b200 import kernels as K

        if self._gate_up is None:
            raise ValueError("prefill_rows needs the fused Llama layer sequence")
        m = self.adapter.hf_model
        layers = m.model.layers
        first = layers[0].input_layernorm
        res, h = K.embed_rmsnorm(m.model.embed_tokens.weight, first.weight,
                                 first.variance_epsilon, tokens)
        last = len(layers) - 1
        for i, layer in enumerate(layers):
            if i == last:
                layer.self_attn._write_kv_rows(h, meta)
                break
            attn = layer.self_attn._prefill_rows(h.unsqueeze(1), meta)
            post = layer.post_attention_layernorm
            K.add_rmsnorm(res, post.weight, post.variance_epsilon, delta=attn.view_as(res), out=h)
            act = K.silu_mul(torch.matmul(h, self._gate_up[i].t()))
            down = layer.mlp.down_proj
            mlp_out = torch.matmul(act, down.weight.t()) if down.bias is None else down(act)
            nxt = layers[i + 1].input_layernorm
            K.add_rmsnorm(res, nxt.weight, nxt.variance_epsilon, delta=mlp_out, out=h)

    @staticmethod
    def padded_rows(rows: int) -> int:
        """GEMM row count of a prefill chunk of ``rows`` rows."""
        return -(-rows // PREFILL_ROW_ALIGN) * PREFILL_ROW_ALIGN

    def warm_prefill_gemms(self, max_rows: int) -> int:
        """Run each prefill GEMM shape once at every padded row count up to
        ``max_rows`` (startup work: cuBLAS then has its kernel choice for all
        of them).  Returns the number of row counts."""
        if self._gate_up is None:
            return 0
        m = self.adapter.hf_model
        d = self.adapter.model_config.d_model
        a0 = m.model.layers[0].self_attn
        nq_d = a0.n_heads * a0.d_k
        down = m.model.layers[0].mlp.down_proj.weight
        top = self.padded_rows(max(1, max_rows))
        # The prefill's operands, same widths (so same leading dimensions).
        zeros = lambda cols: torch.zeros((top, cols), dtype=a0._w_qkv.dtype, device=self.device)
        h, act, attn = zeros(d), zeros(down.shape[1]), zeros(nq_d)
        pairs = [(h, a0._w_qkv), (h, a0._w_qkv[nq_d:]), (h, self._gate_up[0]), (act, down),
                 (attn, a0.W_O.weight)]
        n = 0
        with torch.no_grad():
            for rows in range(PREFILL_ROW_ALIGN, top + 1, PREFILL_ROW_ALIGN):
                for x, w in pairs:
                    torch.matmul(x[:rows], w.t())
                n += 1
        torch.cuda.synchronize(self.device)
        return n

    def _static(self, Bb: int):
        """Static buffers of a bucket:
        [tables Bb x W | lengths | positions | slots | tokens | token sources]."""
        W = self.max_blocks
        n = Bb * W + 5 * Bb
        dev = torch.zeros(n, dtype=torch.int32, device=self.device)
        hosts = [torch.zeros(n, dtype=torch.int32).pin_memory() for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        o = Bb * W
        meta = SimpleNamespace(bt_tensor=dev[:o].view(Bb, W), sl_tensor=dev[o:o + Bb],
                               pos_tensor=dev[o + Bb:o + 2 * Bb],
                               slot_mapping=dev[o + 2 * Bb:o + 3 * Bb])
        vocab = self.adapter.hf_model.lm_head.out_features
        logits = torch.empty((Bb, vocab), dtype=self.adapter.model_config.dtype,
                             device=self.device)
        return SimpleNamespace(Bb=Bb, W=W, dev=dev, hosts=hosts, copied=copied, turn=0,
                               meta=meta, tokens=dev[o + 3 * Bb:o + 4 * Bb],
                               src=dev[o + 4 * Bb:], logits=logits)

    def _stage(self, st, token_ids, seq_ids, positions, seq_lens, src=None) -> None:
        """Pack the batch (padded to the bucket) into pinned memory; one H2D copy."""
        B, Bb, W = len(seq_ids), st.Bb, st.W
        j = st.turn
        st.turn ^= 1
        st.copied[j].synchronize()  # this buffer's previous copy has left it
        host = st.hosts[j]
        h = host.numpy()
        h[:] = 0
        bt = h[:Bb * W].reshape(Bb, W)
        for i, sid in enumerate(seq_ids):
            t = self.kv.get_block_ids(sid)
            bt[i, :len(t)] = t
        o = Bb * W
        pos = np.asarray(positions, dtype=np.int64)
        blk = bt[np.arange(B), pos // self.block_size].astype(np.int64)
        h[o:o + B] = seq_lens
        h[o + Bb:o + Bb + B] = pos
        h[o + 2 * Bb:o + 3 * Bb] = -1  # padding rows own no slot
        h[o + 2 * Bb:o + 2 * Bb + B] = blk * self.block_size + pos % self.block_size
        h[o + 3 * Bb:o + 3 * Bb + B] = token_ids
        h[o + 4 * Bb:] = -1  # host token ids unless a source row is given
        if src is not None:
            h[o + 4 * Bb:o + 4 * Bb + B] = src
        st.dev.copy_(host, non_blocking=True)
        st.copied[j].record()

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
        return all(len(self.kv.get_block_ids(s)) <= self.max_blocks for s in seq_ids)

    def run(self, token_ids, seq_ids, positions, seq_lens, src=None) -> torch.Tensor:
        """Logits ``(B, vocab)`` of one decode step (a view of the bucket's static buffer).

        ``src`` (optional, one int per row): ``src[i] >= 0`` takes row i's
        token from ``prev_tokens[src[i]]`` on the device instead of
        ``token_ids[i]`` (fused Llama path only).
        """
        if src is not None and self._gate_up is None:
            raise ValueError("device-sourced tokens need the fused Llama decode step")
        B = len(seq_ids)
        Bb = self.bucket(B)
        if Bb not in self._graphs:
            self._graphs[Bb] = self._capture(Bb)
        g, st = self._graphs[Bb]
        self._stage(st, token_ids, seq_ids, positions, seq_lens, src)
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
