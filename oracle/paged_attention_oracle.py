"""CPU oracle for the paged decode-attention step -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's CPU path for one decode step
of ``PagedAttentionLayer`` (Nihar0071/vllm_mps).  It is the checker the CUDA
kernels are compared against: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may
import it.  The product path never calls it and has no CPU fallback.

Pinning: every function here is checked against the golden fixtures in
``tests/golden/`` that ``tests/golden/make_golden.py`` produced by running
the reference itself (``tests/test_oracle_golden.py``).

Rounding model.  The reference runs the step in the model dtype (fp16 or
bf16) end to end on the CPU.  PyTorch's CPU kernels for 16-bit floats compute
each op in fp32 and round the result to 16 bits, so the oracle does the same
at the same points:

* RoPE (layers/rotary_embedding.py:13-24, 55-76): cos/sin tables are fp32,
  cast to the model dtype, then ``x*cos`` and ``rotate_half(x)*sin`` are each
  rounded, and so is their sum.
* Attention (layers/paged_attention_layer.py:352-359): ``Q.K^T`` is an fp32
  accumulation rounded to 16 bits, the ``/ sqrt(d_k)`` is rounded again, the
  softmax is computed in fp32 and rounded, and ``P.V`` is an fp32
  accumulation rounded to 16 bits.

The matmul accumulation order inside PyTorch's CPU GEMM is not reproduced,
so a few outputs differ from the reference by one 16-bit ulp; the golden
tests allow 2e-3 absolute + relative, the bar the spec sets.
"""

from __future__ import annotations

import math

import numpy as np

# ── 16-bit float helpers ─────────────────────────────────────────────────────


def bits_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Raw uint16 patterns of ``dtype`` ("float16" | "bfloat16") -> float32."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    raise ValueError(f"unsupported dtype {dtype}")


def f32_to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> raw uint16 of ``dtype`` with round-to-nearest-even."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float16":
        with np.errstate(over="ignore"):  # out-of-range values round to inf, as in torch
            return x.astype(np.float16).view(np.uint16)
    if dtype == "bfloat16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return np.where(nan, np.uint16(0x7FC0), rounded)
    raise ValueError(f"unsupported dtype {dtype}")


def round16(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` and return them as float32."""
    return bits_to_f32(f32_to_bits(x, dtype), dtype)


# ── RoPE (layers/rotary_embedding.py) ────────────────────────────────────────


def rope_inv_freq(d_k: int, theta: float) -> np.ndarray:
    """``1 / theta ** (arange(0, d_k, 2) / d_k)`` in fp32 (rotary_embedding.py:47-49).

    PyTorch's fp32 ``pow`` and numpy's differ in the last bit for some
    entries, so callers that need the reference's exact table pass the one
    built by the product (``vllm_mps_b200.layers.rotary_embedding``) instead.
    """
    e = np.arange(0, d_k, 2, dtype=np.float32) / np.float32(d_k)
    return (np.float32(1.0) / (np.float32(theta) ** e)).astype(np.float32)


def rope_cos_sin(positions: np.ndarray, inv_freq: np.ndarray):
    """fp32 ``cos``/``sin`` rows for each position (rotary_embedding.py:49-53).

    ``freqs = outer(t, inv_freq)`` is one fp32 product per entry; ``emb`` is
    ``cat(freqs, freqs)``.  cos/sin are evaluated in float64 and rounded to
    fp32 (the reference evaluates them in fp32; the two agree to the last
    bit in ~95% of entries and after the cast to 16 bits in >99.99%).
    """
    pos = np.asarray(positions, dtype=np.float32)
    freqs = np.outer(pos, inv_freq.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float64)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """Rotate-half RoPE with the reference's 16-bit rounding points.

    ``x``: float32 values of 16-bit inputs, shape ``(B, H, D)``; ``cos``/``sin``:
    fp32 ``(B, D)``.  Returns float32 values exactly representable in ``dtype``.
    Follows ``apply_rotary`` (rotary_embedding.py:20-24): ``x*cos + rotate_half(x)*sin``
    where ``rotate_half(x) = cat(-x2, x1)`` (:13-17) and cos/sin are cast to
    the tensor dtype first (:71-72).
    """
    c = round16(cos, dtype)[:, None, :]
    s = round16(sin, dtype)[:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = round16(x * c, dtype)
    b = round16(rot * s, dtype)
    return round16(a + b, dtype)


# ── Pool write (memory/mps_memory_pool.py:82-102) ────────────────────────────


def slot_mapping(block_tables, positions, block_size: int):
    """(block_id, token_pos) of each sequence's new token.

    ``block_ids[pos // block_size]``, ``pos % block_size`` as in
    layers/paged_attention_layer.py:318-324 and models/llama_adapter.py:185-193.
    """
    blocks = np.array([int(block_tables[i][p // block_size]) for i, p in enumerate(positions)],
                      dtype=np.int64)
    offs = np.array([int(p) % block_size for p in positions], dtype=np.int64)
    return blocks, offs


def write_kv(pool: np.ndarray, blocks, offs, k_bits, v_bits, num_blocks: int, block_size: int):
    """Write each sequence's K/V rows into ``pool`` (uint16 bits) in place.

    Bounds-checked like ``_validate_indices`` (mps_memory_pool.py:257-268).
    """
    for i, (b, t) in enumerate(zip(blocks, offs)):
        if b < 0 or b >= num_blocks:
            raise IndexError(f"block_id {b} out of range (num_blocks={num_blocks}).")
        if t < 0 or t >= block_size:
            raise IndexError(f"token_pos {t} out of range (block_size={block_size}).")
        pool[b, 0, t] = k_bits[i]
        pool[b, 1, t] = v_bits[i]


# ── Masked softmax attention (layers/paged_attention_layer.py:327-359) ──────


def paged_attention(q_rot: np.ndarray, pool: np.ndarray, block_tables, seq_lens,
                    dtype: str, block_size: int) -> np.ndarray:
    """Decode attention over each sequence's paged K/V history.

    ``q_rot``: float32 values ``(B, n_q, D)``; ``pool``: uint16 bits
    ``(num_blocks, 2, block_size, n_kv, D)``.  Returns float32 values of the
    16-bit output ``(B, n_q, D)``.  Per sequence this is the reference's
    gather of ``seq_len`` slots (:336-343), the GQA head map
    ``kv_head = q_head // (n_q // n_kv)`` (:79-86, :348-350), scores scaled by
    ``1/sqrt(D)`` (:352-353), softmax over the valid slots (:354-355; masked
    slots contribute exactly 0), and the weighted sum of V (:356).
    """
    B, n_q, D = q_rot.shape
    n_kv = pool.shape[3]
    G = n_q // n_kv
    inv = np.float32(1.0 / math.sqrt(D))
    out = np.zeros((B, n_q, D), dtype=np.float32)
    for i in range(B):
        L = int(seq_lens[i])
        if L <= 0:
            continue
        nb = (L + block_size - 1) // block_size
        ids = np.asarray(block_tables[i][:nb], dtype=np.int64)
        kb = pool[ids, 0].reshape(nb * block_size, n_kv, D)[:L]
        vb = pool[ids, 1].reshape(nb * block_size, n_kv, D)[:L]
        K = bits_to_f32(kb, dtype).transpose(1, 0, 2)  # (n_kv, L, D)
        V = bits_to_f32(vb, dtype).transpose(1, 0, 2)
        Kq = np.repeat(K, G, axis=0)  # (n_q, L, D)
        Vq = np.repeat(V, G, axis=0)
        s = round16(np.einsum("hd,hld->hl", q_rot[i], Kq, optimize=True).astype(np.float32), dtype)
        s = round16(s * inv, dtype)
        m = s.max(axis=-1, keepdims=True)
        e = np.exp((s - m).astype(np.float32)).astype(np.float32)
        p = round16(e / e.sum(axis=-1, keepdims=True, dtype=np.float32), dtype)
        o = np.einsum("hl,hld->hd", p, Vq, optimize=True).astype(np.float32)
        out[i] = round16(o, dtype)
    return out


def decode_step(q_bits, k_bits, v_bits, positions, seq_lens, block_tables, pool_bits,
                inv_freq, dtype: str, block_size: int = 16):
    """One reference decode step: RoPE, K/V write, paged attention.

    Mirrors ``PagedAttentionLayer._forward_batch`` between its projections
    (layers/paged_attention_layer.py:275-359).  ``pool_bits`` is updated in
    place.  Returns ``(out_bits (B, n_q, D), k_rot_bits (B, n_kv, D))``.
    """
    q = bits_to_f32(q_bits, dtype)
    k = bits_to_f32(k_bits, dtype)
    cos, sin = rope_cos_sin(np.asarray(positions), inv_freq)
    q_rot = apply_rope(q, cos, sin, dtype)
    k_rot = apply_rope(k, cos, sin, dtype)
    k_rot_bits = f32_to_bits(k_rot, dtype)
    nblk = pool_bits.shape[0]
    blocks, offs = slot_mapping(block_tables, positions, block_size)
    write_kv(pool_bits, blocks, offs, k_rot_bits, np.asarray(v_bits, dtype=np.uint16),
             nblk, block_size)
    out = paged_attention(q_rot, pool_bits, block_tables, seq_lens, dtype, block_size)
    return f32_to_bits(out, dtype), k_rot_bits


def prefill_inputs(seed: int, rows: int, n_q: int, n_kv: int, D: int):
    """Seeded float32 q/k/v of ``rows`` prefill rows (the fixtures' inputs)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((rows, n_q, D), dtype=np.float32)
    k = rng.standard_normal((rows, n_kv, D), dtype=np.float32)
    v = rng.standard_normal((rows, n_kv, D), dtype=np.float32)
    return q, k, v


def prefill(q_bits, k_bits, v_bits, q_start, q_lens, block_tables, pool_bits, inv_freq,
            dtype: str, block_size: int = 16):
    """Causal prefill as the reference computes it: one token at a time.

    Mirrors ``PagedAttentionLayer._forward_single`` (layers/paged_attention_layer.py:175-241)
    called for every prompt token in order: rotate q and k at the token's
    position, write k and v into the token's slot, attend to slots
    ``0..position`` of the sequence.  Rows are laid out sequence after
    sequence (``q_lens[i]`` rows of sequence i at positions
    ``q_start[i] .. q_start[i] + q_lens[i] - 1``).  ``pool_bits`` is updated in
    place.  Returns ``(out_bits (rows, n_q, D), k_rot_bits (rows, n_kv, D))``.
    """
    outs, ks = [], []
    r = 0
    for i, (qs, ql) in enumerate(zip(q_start, q_lens)):
        for t in range(int(ql)):
            pos = int(qs) + t
            o, kr = decode_step(q_bits[r:r + 1], k_bits[r:r + 1], v_bits[r:r + 1], [pos],
                                [pos + 1], [block_tables[i]], pool_bits, inv_freq, dtype,
                                block_size)
            outs.append(o[0])
            ks.append(kr[0])
            r += 1
    n_q, D = q_bits.shape[1], q_bits.shape[2]
    n_kv = k_bits.shape[1]
    if not outs:
        return (np.zeros((0, n_q, D), np.uint16), np.zeros((0, n_kv, D), np.uint16))
    return np.stack(outs), np.stack(ks)
