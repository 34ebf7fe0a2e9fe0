"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

This script is the only place that imports the reference implementation
(Nihar0071/vllm_mps).  It runs the reference's own CPU path and stores its
inputs and outputs as small ``.npz`` files, which the tests then compare both
the CPU oracle and the CUDA kernels against.  It needs the reference source
tree (pass ``--ref``); the fixtures it writes are committed so that nothing
at test time needs the reference.

What is captured
----------------
* ``attn_*.npz`` -- one ``PagedAttentionLayer._forward_batch`` call
  (layers/paged_attention_layer.py:245-364) with the Metal branch switched
  off, i.e. the reference's Python fallback at :316-359.  The layer's
  projections are replaced by fixed tensors so that q/k/v are exactly the
  seeded N(0,1) values the benchmark configs describe; the input of ``W_O``
  (the attention output, :358-362) is captured.  The memory pool is
  regenerated from a seed (numpy PCG64) and only the slots the step wrote
  are stored.
* ``slots_trace.npz`` -- a seeded random op stream (allocate, append_slot,
  free, fork, swap_out, swap_in) through the reference ``KVCacheManager``
  (core/kv_cache_manager.py:21-298) with the block table of every live
  sequence and the free counts after every op.
* ``sched_trace.npz`` -- a seeded request stream through the reference
  ``Scheduler`` (engine/scheduler.py:86-226): per step the scheduled
  sequence ids, the preempted groups and every block table.
* ``prefill_*.npz`` -- prompt rows through the reference's single-token
  path (layers/paged_attention_layer.py:175-241), token by token: the oracle
  of the causal prefill kernel.  Inputs are regenerated from ``input_seed``
  (``prefill_inputs``), the pool from ``pool_seed``.
* ``engine_c0.npz`` -- config 0 end to end: the TinyLlama-shaped random
  fp16 model (seed 0), 8 prompts x 32 ids, 20 greedy steps through the
  reference engine (engine/llm_engine.py:316-346); tokens plus the top-5
  logits of every decision, and the shared pool's used blocks at the start
  of decisions 5 and 14.  (Needs ~2 min of CPU; ``--skip-engine``.)
* ``engine_c0_physical.npz`` -- the same model and prompts through the
  reference's classes with one pool per layer and every prompt token but
  the last run through the single-token path first (the well-conditioned
  mode), then 20 greedy steps of the reference engine.

Usage::

    python tests/golden/make_golden.py --ref /path/to/vllm_mps
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# name, n_q, n_kv, D, dtype, B, ctx_lo, ctx_hi, num_blocks, theta, max_pos, seed, explicit ctx list
ATTN_CASES = [
    ("attn_c1_small", 32, 4, 64, "float16", 8, 1, 300, 192, 10000.0, 2048, 11, None),
    ("attn_c1_edges", 32, 4, 64, "float16", 9, 1, 1, 96, 10000.0, 2048, 12,
     [1, 2, 15, 16, 17, 31, 32, 33, 48]),
    ("attn_c1_b1", 32, 4, 64, "float16", 1, 700, 700, 64, 10000.0, 2048, 13, None),
    ("attn_c2_small", 32, 8, 128, "bfloat16", 4, 100, 600, 160, 500000.0, 8192, 14, None),
    ("attn_c3_small", 64, 8, 128, "float16", 2, 900, 1500, 200, 10000.0, 4096, 15, None),
    ("attn_mha_small", 8, 8, 64, "float16", 3, 1, 90, 32, 10000.0, 2048, 16, None),
    ("attn_g2_small", 16, 8, 64, "float16", 5, 1, 150, 64, 10000.0, 2048, 17, None),
]


def import_reference(ref_path: str):
    """Import the reference as package ``vllm_mps`` and switch its Metal branch off.

    The Metal kernel needs ``torch.mps.compile_shader`` (kernels/__init__.py:255,
    262), which does not exist off Apple hardware, and the switch is a local
    constant (layers/paged_attention_layer.py:289).  Re-executing the module
    source with that one line flipped runs the reference's own fallback.
    """
    tmp = tempfile.mkdtemp(prefix="vmps_ref_")
    os.symlink(os.path.abspath(ref_path), os.path.join(tmp, "vllm_mps"))
    sys.path.insert(0, tmp)
    import vllm_mps.layers.paged_attention_layer as pal

    src = open(pal.__file__).read()
    assert src.count("use_metal_kernel = True") == 1
    src = src.replace("use_metal_kernel = True", "use_metal_kernel = False")
    exec(compile(src, pal.__file__, "exec"), pal.__dict__)
    return pal


def pool_from_seed(seed: int, shape, dtype_name: str) -> np.ndarray:
    """Seeded N(0,1) pool contents as raw 16-bit patterns (uint16)."""
    import torch

    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=shape, dtype=np.float32)
    t = torch.from_numpy(x).to(getattr(torch, dtype_name))
    return t.view(torch.int16).numpy().view(np.uint16)


def to_bits(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(bits: np.ndarray, dtype_name: str):
    import torch

    return torch.from_numpy(bits.view(np.int16).copy()).view(getattr(torch, dtype_name))


def gen_attn_case(pal, case):
    import torch
    import torch.nn as nn
    from vllm_mps.core.model_config import ModelConfig
    from vllm_mps.memory.mps_memory_pool import MPSMemoryPool

    (name, n_q, n_kv, D, dtn, B, lo, hi, nblk, theta, max_pos, seed, ctx_list) = case
    dt = getattr(torch, dtn)
    bs = 16
    rng = np.random.default_rng(seed)
    if ctx_list is not None:
        ctx = np.array(ctx_list, dtype=np.int64)
    else:
        ctx = rng.integers(lo, hi + 1, size=B)
    pages = (ctx + bs - 1) // bs
    assert pages.sum() <= nblk, (name, pages.sum(), nblk)
    perm = rng.permutation(nblk)
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off: off + p]])
        off += p
    max_blocks = int(pages.max())
    bt = np.zeros((B, max_blocks), dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = t

    q = rng.standard_normal((B, n_q, D), dtype=np.float32)
    k = rng.standard_normal((B, n_kv, D), dtype=np.float32)
    v = rng.standard_normal((B, n_kv, D), dtype=np.float32)
    q_t = torch.from_numpy(q).to(dt)
    k_t = torch.from_numpy(k).to(dt)
    v_t = torch.from_numpy(v).to(dt)

    pool_seed = seed * 1000 + 7
    pshape = (nblk, 2, bs, n_kv, D)
    pool_bits = pool_from_seed(pool_seed, pshape, dtn)

    cfg = ModelConfig(
        model_name="synthetic", architecture="llama", d_model=n_q * D,
        n_heads=n_q, n_kv_heads=n_kv, d_k=D, n_layers=1, vocab_size=32000,
        max_seq_len=max_pos, rope_theta=theta, dtype=dt,
        device=torch.device("cpu"),
    )
    pool = MPSMemoryPool(nblk, bs, n_kv, D, dt, torch.device("cpu"))
    pool._pool.copy_(from_bits(pool_bits, dtn).view(pshape))

    class _Tables:
        def get_block_table(self, seq_id):
            return tables[seq_id]

    class _Fixed(nn.Module):
        def __init__(self, t):
            super().__init__()
            self.t = t

        def forward(self, x):
            return self.t

    captured = {}

    class _Capture(nn.Module):
        def forward(self, x):
            captured["attn_out"] = x.detach().clone()
            return x

    rot = pal.RotaryEmbedding(D, max_pos, theta, torch.device("cpu"))
    layer = pal.PagedAttentionLayer(
        0, cfg, _Tables(), pool,
        _Fixed(q_t.reshape(B, 1, n_q * D)),
        _Fixed(k_t.reshape(B, 1, n_kv * D)),
        _Fixed(v_t.reshape(B, 1, n_kv * D)),
        _Capture(), rot,
    )
    positions = [int(c) - 1 for c in ctx]
    seq_lens = [int(c) for c in ctx]
    hidden = torch.zeros(B, 1, n_q * D, dtype=dt)
    with torch.no_grad():
        layer._forward_batch(hidden, list(range(B)), positions, seq_lens)
    out = captured["attn_out"].reshape(B, n_q, D)

    # Slot mapping the reference used (layers/paged_attention_layer.py:318-324).
    slot_block = np.array([tables[i][positions[i] // bs] for i in range(B)], dtype=np.int32)
    slot_off = np.array([positions[i] % bs for i in range(B)], dtype=np.int32)
    new_pool = pool._pool
    written_k = torch.stack([new_pool[slot_block[i], 0, slot_off[i]] for i in range(B)])
    written_v = torch.stack([new_pool[slot_block[i], 1, slot_off[i]] for i in range(B)])

    # All other slots must be untouched.
    before = from_bits(pool_bits, dtn).view(pshape).clone()
    for i in range(B):
        before[slot_block[i], 0, slot_off[i]] = new_pool[slot_block[i], 0, slot_off[i]]
        before[slot_block[i], 1, slot_off[i]] = new_pool[slot_block[i], 1, slot_off[i]]
    assert torch.equal(before.view(torch.int16), new_pool.view(torch.int16))

    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        n_q=n_q, n_kv=n_kv, D=D, dtype=dtn, block_size=bs, num_blocks=nblk,
        theta=theta, max_pos=max_pos, pool_seed=pool_seed,
        pool_sha256=hashlib.sha256(pool_bits.tobytes()).hexdigest(),
        seq_lens=np.array(seq_lens, dtype=np.int32),
        positions=np.array(positions, dtype=np.int32),
        block_tables=bt,
        q=to_bits(q_t), k=to_bits(k_t), v=to_bits(v_t),
        slot_block=slot_block, slot_off=slot_off,
        written_k=to_bits(written_k), written_v=to_bits(written_v),
        attn_out=to_bits(out),
        cos_at_pos=rot.cos_cached[positions].numpy(),
        sin_at_pos=rot.sin_cached[positions].numpy(),
    )
    print(f"{name}: B={B} ctx={list(map(int, ctx))[:6]}... written")


# name, n_q, n_kv, D, dtype, [(q_start, q_len) per sequence], num_blocks, theta, max_pos, seed
PREFILL_CASES = [
    ("prefill_c1", 32, 4, 64, "float16", [(0, 37), (20, 30), (130, 6)], 40, 10000.0, 2048, 21),
    ("prefill_c2", 16, 4, 128, "bfloat16", [(0, 33), (33, 12)], 24, 500000.0, 8192, 22),
    ("prefill_mha", 4, 4, 64, "float16", [(0, 130), (7, 1)], 24, 10000.0, 2048, 23),
    ("prefill_g16", 32, 2, 64, "float16", [(0, 24), (17, 9)], 16, 10000.0, 2048, 24),
]


def prefill_inputs(seed, rows, n_q, n_kv, D):
    """Seeded float32 q/k/v of every prefill row (the tests regenerate them)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((rows, n_q, D), dtype=np.float32)
    k = rng.standard_normal((rows, n_kv, D), dtype=np.float32)
    v = rng.standard_normal((rows, n_kv, D), dtype=np.float32)
    return q, k, v


def gen_prefill_case(pal, case):
    """Prompt rows through the reference's single-token path, token by token.

    ``_forward_single`` (layers/paged_attention_layer.py:175-241) writes the
    token's rotated K and V into its slot, then attends to the sequence's
    slots ``0..position`` -- per token, the causal prefill that kernel 3 does
    for a whole prompt at once.  Sequence i already holds ``q_start`` tokens
    (the seeded pool contents); its ``q_len`` new rows follow in order.
    """
    import torch
    import torch.nn as nn
    from vllm_mps.core.model_config import ModelConfig
    from vllm_mps.memory.mps_memory_pool import MPSMemoryPool

    (name, n_q, n_kv, D, dtn, seqs, nblk, theta, max_pos, seed) = case
    dt = getattr(torch, dtn)
    bs = 16
    rng = np.random.default_rng(seed)
    ctx = [qs + ql for qs, ql in seqs]
    pages = [(c + bs - 1) // bs for c in ctx]
    assert sum(pages) <= nblk, (name, pages, nblk)
    perm = rng.permutation(nblk)
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off: off + p]])
        off += p
    bt = np.zeros((len(seqs), max(pages)), dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = t
    rows = sum(ql for _, ql in seqs)
    q32, k32, v32 = prefill_inputs(seed * 1000 + 1, rows, n_q, n_kv, D)
    q_t, k_t, v_t = (torch.from_numpy(x).to(dt) for x in (q32, k32, v32))

    pool_seed = seed * 1000 + 7
    pshape = (nblk, 2, bs, n_kv, D)
    pool_bits = pool_from_seed(pool_seed, pshape, dtn)
    cfg = ModelConfig(
        model_name="synthetic", architecture="llama", d_model=n_q * D,
        n_heads=n_q, n_kv_heads=n_kv, d_k=D, n_layers=1, vocab_size=32000,
        max_seq_len=max_pos, rope_theta=theta, dtype=dt, device=torch.device("cpu"),
    )
    pool = MPSMemoryPool(nblk, bs, n_kv, D, dt, torch.device("cpu"))
    pool._pool.copy_(from_bits(pool_bits, dtn).view(pshape))

    class _Tables:
        def get_block_table(self, seq_id):
            return tables[seq_id]

    cur = {"row": 0}

    class _Row(nn.Module):
        def __init__(self, t, width):
            super().__init__()
            self.t, self.width = t, width

        def forward(self, x):
            return self.t[cur["row"]].reshape(1, 1, self.width)

    outs = []

    class _Capture(nn.Module):
        def forward(self, x):
            outs.append(x.detach().clone().reshape(n_q, D))
            return x

    rot = pal.RotaryEmbedding(D, max_pos, theta, torch.device("cpu"))
    layer = pal.PagedAttentionLayer(
        0, cfg, _Tables(), pool, _Row(q_t, n_q * D), _Row(k_t, n_kv * D), _Row(v_t, n_kv * D),
        _Capture(), rot,
    )
    q_start = np.array([qs for qs, _ in seqs], dtype=np.int32)
    q_lens = np.array([ql for _, ql in seqs], dtype=np.int32)
    hidden = torch.zeros(1, 1, n_q * D, dtype=dt)
    written_k = []
    with torch.no_grad():
        for i, (qs, ql) in enumerate(seqs):
            for t in range(ql):
                pos = qs + t
                layer.set_context(i, pos)
                layer._forward_single(hidden)
                written_k.append(pool._pool[tables[i][pos // bs], 0, pos % bs].clone())
                cur["row"] += 1
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        n_q=n_q, n_kv=n_kv, D=D, dtype=dtn, block_size=bs, num_blocks=nblk,
        theta=theta, max_pos=max_pos, pool_seed=pool_seed, input_seed=seed * 1000 + 1,
        pool_sha256=hashlib.sha256(pool_bits.tobytes()).hexdigest(),
        q_start=q_start, q_lens=q_lens, block_tables=bt,
        written_k=to_bits(torch.stack(written_k)), attn_out=to_bits(torch.stack(outs)),
    )
    print(f"{name}: rows={rows} written")


def gen_slots_trace():
    """Random op stream through the reference KVCacheManager (bit-exact slotting)."""
    from vllm_mps.core.kv_cache_manager import KVCacheManager

    rng = np.random.default_rng(2024)
    gpu, cpu = 48, 24
    m = KVCacheManager(gpu, cpu)
    live, swapped = [], []
    next_id = 0
    ops, args, tables_out, free_out = [], [], [], []
    for step in range(600):
        r = rng.random()
        if r < 0.15 or not live:
            m.allocate(next_id)
            live.append(next_id)
            op, a = "allocate", (next_id, -1)
            next_id += 1
        elif r < 0.70:
            s = live[rng.integers(len(live))]
            n = int(rng.integers(1, 20))
            done = 0
            try:
                for _ in range(n):
                    m.append_slot(s)
                    done += 1
                op = "append"
            except MemoryError:
                op = "append_oom"
            a = (s, done)
        elif r < 0.80:
            s = live.pop(rng.integers(len(live)))
            m.free(s)
            op, a = "free", (s, -1)
        elif r < 0.87:
            s = live[rng.integers(len(live))]
            m.fork(s, next_id)
            live.append(next_id)
            op, a = "fork", (s, next_id)
            next_id += 1
        elif r < 0.94:
            s = live[rng.integers(len(live))]
            # Only forked-free tables swap cleanly (swap_out frees shared blocks
            # once per owner); require enough CPU blocks and sole ownership.
            blocks = m._block_tables[s]._blocks
            if len(blocks) > m.get_num_free_cpu_blocks() or any(b.ref_count != 1 for b in blocks):
                continue
            live.remove(s)
            m.swap_out(s)
            swapped.append(s)
            op, a = "swap_out", (s, -1)
        elif swapped:
            s = swapped[0]
            if len(m._block_tables[s]._blocks) > m.get_num_free_gpu_blocks():
                continue
            swapped.pop(0)
            m.swap_in(s)
            live.append(s)
            op, a = "swap_in", (s, -1)
        else:
            continue
        if m.get_num_free_gpu_blocks() == 0 and rng.random() < 0.5:
            # Keep the stream going: record this op, then release the oldest
            # live sequence as an op of its own.
            ops.append(op)
            args.append(a)
            snap = {q: m.get_block_table(q) for q in sorted(m.get_all_seq_ids())}
            tables_out.append(repr(snap))
            free_out.append((m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()))
            s = live.pop(0)
            m.free(s)
            op, a = "free", (s, -1)
        ops.append(op)
        args.append(a)
        snap = {q: m.get_block_table(q) for q in sorted(m.get_all_seq_ids())}
        tables_out.append(repr(snap))
        free_out.append((m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()))
    np.savez_compressed(
        os.path.join(HERE, "slots_trace.npz"),
        gpu=gpu, cpu=cpu, ops=np.array(ops), args=np.array(args, dtype=np.int64),
        tables=np.array(tables_out), free=np.array(free_out, dtype=np.int64),
    )
    print(f"slots_trace: {len(ops)} ops written")


def gen_sched_trace(seed: int = 77, gpu: int = 40, out_name: str = "sched_trace.npz"):
    """Seeded request stream through the reference Scheduler."""
    from vllm_mps.core.kv_cache_manager import KVCacheManager
    from vllm_mps.core.sequence import SamplingParams, Sequence, SequenceGroup, SequenceStatus
    from vllm_mps.engine.scheduler import Scheduler

    rng = np.random.default_rng(seed)
    kv = KVCacheManager(gpu, 40)
    sched = Scheduler(kv, max_batch_size=6, max_tokens_per_step=300)
    reqs = []
    for i in range(24):
        plen = int(rng.integers(1, 60))
        mx = int(rng.integers(1, 40))
        reqs.append((i, plen, mx))
    pending = list(reqs)
    groups = {}
    steps = []
    for step in range(400):
        # Arrivals: up to 2 new requests per step.
        for _ in range(int(rng.integers(0, 3))):
            if pending:
                gid, plen, mx = pending.pop(0)
                p = SamplingParams(temperature=0.0, max_tokens=mx)
                g = SequenceGroup(gid, [Sequence(gid, "", list(range(plen)), p)], p)
                groups[gid] = g
                sched.add_request(g)
        try:
            out = sched.schedule()
        except MemoryError as e:
            # The reference checks can_allocate(seq, 1) per group, not
            # cumulatively (engine/scheduler.py:163-196), so step 4 can still
            # run out of blocks.  Record it; the trace ends there.
            steps.append(repr(("MemoryError", str(e))))
            break
        scheduled = [s.seq_id for g in out.scheduled_groups for s in g.get_seqs(SequenceStatus.RUNNING)]
        preempted = [g.group_id for g in out.preempted_groups]
        tables = {s: kv.get_block_table(s) for s in sorted(kv.get_all_seq_ids())}
        # Emulate the engine: every scheduled seq gets one token (id = step).
        for g in out.scheduled_groups:
            for s in g.get_seqs(SequenceStatus.RUNNING):
                s.add_token(step % 1000)
                if s.is_finished():
                    sched.mark_finished(s.seq_id)
        steps.append(repr((scheduled, preempted, out.num_batched_tokens,
                           out.num_scheduled_seqs, tables,
                           sched.get_num_waiting(), sched.get_num_running(),
                           sched.get_num_preempted())))
        if not pending and sched.get_num_waiting() == 0 and sched.get_num_running() == 0 \
                and sched.get_num_preempted() == 0:
            break
    np.savez_compressed(
        os.path.join(HERE, out_name),
        reqs=np.array(reqs, dtype=np.int64), steps=np.array(steps),
        gpu=gpu, cpu=40, max_batch=6, max_tokens=300, arrival_seed=seed,
    )
    print(f"sched_trace: {len(steps)} steps written")


def c0_llama_config():
    from transformers import LlamaConfig

    return LlamaConfig(
        hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
        num_attention_heads=32, num_key_value_heads=4, vocab_size=32000,
        rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048,
        tie_word_embeddings=False,
    )


# Decisions of the config-0 run at whose start the pool is recorded: a
# restart point for one-step checks (the shared-pool trace amplifies rounding
# differences from step to step, so later steps are compared from here).
C0_SNAP_STEPS = (5, 14)


def gen_engine_c0(pal):
    """Config 0 through the reference engine, CPU fp16, greedy, 20 steps."""
    import torch
    from transformers import LlamaForCausalLM
    from vllm_mps.core.kv_cache_manager import KVCacheManager
    from vllm_mps.core.model_config import ModelConfig
    from vllm_mps.core.sequence import SamplingParams, Sequence, SequenceGroup
    from vllm_mps.engine.llm_engine import LLMEngine, RequestOutput
    from vllm_mps.engine.scheduler import Scheduler
    from vllm_mps.memory.mps_memory_pool import MPSMemoryPool
    from vllm_mps.model.sampler import Sampler
    import vllm_mps.models.llama_adapter as la

    torch.set_num_threads(os.cpu_count())
    hf_cfg = c0_llama_config()
    torch.manual_seed(0)
    model = LlamaForCausalLM(hf_cfg).to(torch.float16).eval()
    cfg = ModelConfig(
        model_name="tinyllama-random", architecture="llama", d_model=2048,
        n_heads=32, n_kv_heads=4, d_k=64, n_layers=22, vocab_size=32000,
        max_seq_len=2048, rope_theta=10000.0, dtype=torch.float16,
        device=torch.device("cpu"),
    )
    pool = MPSMemoryPool(256, 16, 4, 64, torch.float16, torch.device("cpu"))
    kv = KVCacheManager(256, 128)
    adapter = la.LlamaAdapter("tinyllama-random")
    adapter.model_config, adapter.kv_cache_manager, adapter.memory_pool = cfg, kv, pool
    adapter.hf_model = model
    adapter.paged_layers = []
    for i, layer in enumerate(model.model.layers):
        pl = pal.PagedAttentionLayer.from_llama_layer(layer.self_attn, i, cfg, kv, pool)
        layer.self_attn = pl
        adapter.paged_layers.append(pl)

    eng = LLMEngine.__new__(LLMEngine)
    eng.memory_pool, eng.kv_cache_manager = pool, kv
    eng.scheduler = Scheduler(kv, max_batch_size=8, max_tokens_per_step=100000)
    eng.sampler = Sampler()
    eng.model = eng.model_runner = None
    eng._request_counter = 0
    eng._outputs, eng._seq_to_request, eng._seq_to_params = {}, {}, {}
    eng.total_tokens_generated = 0
    eng.start_time = time.time()
    eng.adapter = adapter
    eng.model_config = cfg

    class _Tok:
        def decode(self, ids, skip_special_tokens=True):
            return ""

    eng.tokenizer = _Tok()
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, 32000, (8, 32), generator=g).tolist()
    params = SamplingParams(temperature=0.0, max_tokens=20)
    for rid, p in enumerate(prompts):
        seq = Sequence(rid, "", p, params)
        eng.scheduler.add_request(SequenceGroup(rid, [seq], params))
        eng._outputs[rid] = RequestOutput(request_id=rid, prompt="")
        eng._seq_to_request[rid] = rid
        eng._seq_to_params[rid] = params

    # Record the top-5 logits of each decision by wrapping forward_batch.
    top_vals, top_ids, step_seqs = [], [], []
    orig = adapter.forward_batch

    snaps = {}

    def wrapped(token_ids, seq_ids, positions, seq_lens):
        step = len(top_vals)
        if step in C0_SNAP_STEPS:
            # Pool contents at the start of this decision (before any layer
            # writes), restricted to the blocks the running sequences own.
            ids = sorted({b for sid in seq_ids for b in kv.get_block_table(sid)})
            snaps[step] = (np.array(ids, dtype=np.int64),
                           pool._pool[ids].contiguous().view(torch.int16).numpy().view(np.uint16))
        logits = orig(token_ids, seq_ids, positions, seq_lens)
        v, i = torch.topk(logits.float(), 5, dim=-1)
        top_vals.append(v.numpy())
        top_ids.append(i.numpy())
        step_seqs.append(list(seq_ids))
        return logits

    adapter.forward_batch = wrapped
    t0 = time.perf_counter()
    steps = 0
    while not eng.is_finished():
        eng.step()
        steps += 1
    dt = time.perf_counter() - t0
    tokens = np.array([eng._outputs[r].token_ids for r in range(8)], dtype=np.int64)
    np.savez_compressed(
        os.path.join(HERE, "engine_c0.npz"),
        prompts=np.array(prompts, dtype=np.int64), tokens=tokens,
        top_vals=np.stack(top_vals), top_ids=np.stack(top_ids),
        step_seqs=np.array(step_seqs, dtype=np.int64),
        cpu_seconds=dt, cpu_threads=torch.get_num_threads(),
        snap_steps=np.array(sorted(snaps), dtype=np.int64),
        **{f"snap{t}_blocks": snaps[t][0] for t in snaps},
        **{f"snap{t}_pool": snaps[t][1] for t in snaps},
    )
    print(f"engine_c0: {steps} steps, {tokens.size} tokens in {dt:.2f}s")


def gen_engine_c0_physical(pal, steps: int = 20):
    """Config 0 through the reference classes in the well-conditioned mode.

    The reference engine shares ONE pool across all layers and feeds only
    the last prompt token (engine/llm_engine.py:166-193, :323-329), which
    makes its trace chaotic under rounding.  Its layer takes the pool as a
    constructor argument (layers/paged_attention_layer.py:36-38), so here
    every layer gets its own ``MPSMemoryPool``; after the first
    ``Scheduler.schedule()`` has allocated the prompt slots, every prompt
    token but the last is run through the single-token path
    (``LlamaAdapter.forward_single_token``, models/llama_adapter.py:112-133 ->
    ``_forward_single``, layers/paged_attention_layer.py:175-241), in order,
    so each layer's pool holds the prompt's K/V; then ``steps`` greedy decode
    steps run through the reference engine (``_step_adapter`` for the
    first, ``step()`` after it).  Stored: tokens, top-5 logits and ids of
    every decision.
    """
    import torch
    from transformers import LlamaForCausalLM
    from vllm_mps.core.kv_cache_manager import KVCacheManager
    from vllm_mps.core.model_config import ModelConfig
    from vllm_mps.core.sequence import SamplingParams, Sequence, SequenceGroup
    from vllm_mps.engine.llm_engine import LLMEngine, RequestOutput
    from vllm_mps.engine.scheduler import Scheduler
    from vllm_mps.memory.mps_memory_pool import MPSMemoryPool
    from vllm_mps.model.sampler import Sampler
    import vllm_mps.models.llama_adapter as la

    torch.set_num_threads(os.cpu_count())
    hf_cfg = c0_llama_config()
    torch.manual_seed(0)
    model = LlamaForCausalLM(hf_cfg).to(torch.float16).eval()
    cfg = ModelConfig(
        model_name="tinyllama-random", architecture="llama", d_model=2048,
        n_heads=32, n_kv_heads=4, d_k=64, n_layers=22, vocab_size=32000,
        max_seq_len=2048, rope_theta=10000.0, dtype=torch.float16,
        device=torch.device("cpu"),
    )
    nblocks = 64
    kv = KVCacheManager(nblocks, 32)
    pools = [MPSMemoryPool(nblocks, 16, 4, 64, torch.float16, torch.device("cpu"))
             for _ in model.model.layers]
    adapter = la.LlamaAdapter("tinyllama-random")
    adapter.model_config, adapter.kv_cache_manager, adapter.memory_pool = cfg, kv, pools[0]
    adapter.hf_model = model
    adapter.paged_layers = []
    for i, layer in enumerate(model.model.layers):
        pl = pal.PagedAttentionLayer.from_llama_layer(layer.self_attn, i, cfg, kv, pools[i])
        layer.self_attn = pl
        adapter.paged_layers.append(pl)

    eng = LLMEngine.__new__(LLMEngine)
    eng.memory_pool, eng.kv_cache_manager = pools[0], kv
    eng.scheduler = Scheduler(kv, max_batch_size=8, max_tokens_per_step=100000)
    eng.sampler = Sampler()
    eng.model = eng.model_runner = None
    eng._request_counter = 0
    eng._outputs, eng._seq_to_request, eng._seq_to_params = {}, {}, {}
    eng.total_tokens_generated = 0
    eng.start_time = time.time()
    eng.adapter = adapter
    eng.model_config = cfg

    class _Tok:
        def decode(self, ids, skip_special_tokens=True):
            return ""

    eng.tokenizer = _Tok()
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, 32000, (8, 32), generator=g).tolist()
    params = SamplingParams(temperature=0.0, max_tokens=steps)
    for rid, p in enumerate(prompts):
        seq = Sequence(rid, "", p, params)
        eng.scheduler.add_request(SequenceGroup(rid, [seq], params))
        eng._outputs[rid] = RequestOutput(request_id=rid, prompt="")
        eng._seq_to_request[rid] = rid
        eng._seq_to_params[rid] = params

    top_vals, top_ids, step_seqs = [], [], []
    orig = adapter.forward_batch

    def wrapped(token_ids, seq_ids, positions, seq_lens):
        logits = orig(token_ids, seq_ids, positions, seq_lens)
        v, i = torch.topk(logits.float(), 5, dim=-1)
        top_vals.append(v.numpy())
        top_ids.append(i.numpy())
        step_seqs.append(list(seq_ids))
        return logits

    adapter.forward_batch = wrapped
    t0 = time.perf_counter()
    sched_out = eng.scheduler.schedule()  # admits all 8, allocates the prompt slots
    assert len(sched_out.scheduled_groups) == 8
    for rid, p in enumerate(prompts):
        for pos, tok in enumerate(p[:-1]):
            adapter.forward_single_token(tok, pos, rid)
    t_prefill = time.perf_counter() - t0
    eng._step_adapter(sched_out)
    n = 1
    while not eng.is_finished():
        eng.step()
        n += 1
    dt = time.perf_counter() - t0
    tokens = np.array([eng._outputs[r].token_ids for r in range(8)], dtype=np.int64)
    np.savez_compressed(
        os.path.join(HERE, "engine_c0_physical.npz"),
        prompts=np.array(prompts, dtype=np.int64), tokens=tokens,
        top_vals=np.stack(top_vals), top_ids=np.stack(top_ids),
        step_seqs=np.array(step_seqs, dtype=np.int64),
        cpu_seconds=dt, prefill_seconds=t_prefill, cpu_threads=torch.get_num_threads(),
    )
    print(f"engine_c0_physical: {n} steps, {tokens.size} tokens in {dt:.1f}s "
          f"(prefill {t_prefill:.1f}s)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference source tree")
    ap.add_argument("--skip-engine", action="store_true")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    pal = import_reference(a.ref)
    for case in ATTN_CASES:
        if not a.only or a.only in case[0]:
            gen_attn_case(pal, case)
    for case in PREFILL_CASES:
        if not a.only or a.only in case[0]:
            gen_prefill_case(pal, case)
    if not a.only or a.only == "slots":
        gen_slots_trace()
    if not a.only or a.only == "sched":
        # Seed 76 on 40 blocks preempts and resumes and then drains; seed 74
        # on 48 blocks preempts three times and ends in the reference's
        # step-4 MemoryError.
        gen_sched_trace(76, 40, "sched_trace.npz")
        gen_sched_trace(74, 48, "sched_trace_oom.npz")
    if not a.skip_engine and (not a.only or a.only == "engine"):
        gen_engine_c0(pal)
    if not a.skip_engine and (not a.only or a.only == "engine_physical"):
        gen_engine_c0_physical(pal)


if __name__ == "__main__":
    main()
