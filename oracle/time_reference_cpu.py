"""Times the reference's OWN CPU decode path on the config-1 workload (test infrastructure).

The reference (Nihar0071/vllm_mps) is Python; off Apple hardware its decode
attention is the fallback of ``PagedAttentionLayer._forward_batch``
(layers/paged_attention_layer.py:316-359: per-sequence RoPE, write_kv and
block gather loops, padding, the GQA repeat, fp16 softmax attention).  It
cannot travel to the GPU box (the box has no copy of the reference), so this
script runs it where the reference source is, on the same seeded config-1
workload that ``bench.py`` times (64 sequences, contexts from
``bench.make_host_workload`` with the bench's seed, 32/4 heads, head_dim 64,
fp16, a 16384-block pool), with every host thread, and prints one JSON line:
tokens/s and milliseconds per decode step of one layer.  Its result is quoted
beside the C port that ``bench.py --impl reference`` times on the GPU box's
host (``oracle/vmps_oracle.c``).

Usage::

    python oracle/time_reference_cpu.py --ref <reference source tree> [--steps 5]
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--steps", type=int, default=5)
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import torch
    import torch.nn as nn

    import bench
    from make_golden import import_reference

    pal = import_reference(a.ref)
    from vllm_mps.core.model_config import ModelConfig
    from vllm_mps.memory.mps_memory_pool import MPSMemoryPool

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = bench.CONFIGS["c1"]
    B, n_q, n_kv, D, dtn, lo, hi, nb, R, desc = cfg
    ctx, pages, tables = bench.make_host_workload(cfg, seed=1000)
    dt = getattr(torch, dtn)
    g = torch.Generator().manual_seed(99)
    pool = MPSMemoryPool(nb, 16, n_kv, D, dt, torch.device("cpu"))
    pool._pool.copy_(torch.randn(pool._pool.shape, generator=g).to(dt))
    q = torch.randn(B, 1, n_q * D, generator=g).to(dt)
    k = torch.randn(B, 1, n_kv * D, generator=g).to(dt)
    v = torch.randn(B, 1, n_kv * D, generator=g).to(dt)
    mcfg = ModelConfig(model_name="c1", architecture="llama", d_model=n_q * D, n_heads=n_q,
                       n_kv_heads=n_kv, d_k=D, n_layers=1, vocab_size=32000, max_seq_len=2048,
                       rope_theta=10000.0, dtype=dt, device=torch.device("cpu"))

    class _Tables:
        def __init__(self, t):
            self.t = t

        def get_block_table(self, seq_id):
            return [int(x) for x in self.t[seq_id, :pages[seq_id]]]

    class _Fixed(nn.Module):
        def __init__(self, t):
            super().__init__()
            self.t = t

        def forward(self, x):
            return self.t

    rot = pal.RotaryEmbedding(D, 2048, 10000.0, torch.device("cpu"))
    layers = [pal.PagedAttentionLayer(0, mcfg, _Tables(t), pool, _Fixed(q), _Fixed(k), _Fixed(v),
                                      nn.Identity(), rot) for t in tables]
    positions = [int(c) - 1 for c in ctx]
    seq_lens = [int(c) for c in ctx]
    hidden = torch.zeros(B, 1, n_q * D, dtype=dt)
    with torch.no_grad():
        layers[0]._forward_batch(hidden, list(range(B)), positions, seq_lens)  # warm-up
        t0 = time.perf_counter()
        for i in range(a.steps):
            layers[i % R]._forward_batch(hidden, list(range(B)), positions, seq_lens)
        el = time.perf_counter() - t0
    print(json.dumps({
        "what": "reference CPU decode path (layers/paged_attention_layer.py:316-359), config 1",
        "workload": desc, "sum_ctx": int(ctx.sum()), "steps": a.steps,
        "ms_per_step": el / a.steps * 1e3, "tokens_per_s": B * a.steps / el,
        "threads": torch.get_num_threads(), "cpu_count": os.cpu_count(),
        "torch": torch.__version__,
    }))


if __name__ == "__main__":
    main()
