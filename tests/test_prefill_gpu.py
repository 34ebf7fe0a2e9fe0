"""Parity of the tcgen05 causal prefill kernel (kernel 3) through the C ABI.

Checks, on a B200:
* against the reference's own outputs (``tests/golden/prefill_*.npz``: the
  prompt rows run through the reference's single-token path, token by
  token): kernel 1 writes every row's K/V bit-exact, kernel 3's outputs are
  within 2e-3 absolute + relative (bf16: two bf16 ulps at magnitude 1 and
  99.9 % within one, because the reference rounds Q.K^T and P to bf16);
* against a PyTorch fp32 causal attention (2e-3; bf16 2^-7) over the same pool on larger
  seeded cases: several key tiles and query tiles, a cached prefix
  (q_start > 0), G = 1, 2, 4, 8, 16, head_dim 64 and 128, fp16 and bf16,
  a zero-length sequence, strided q rows;
* against the decode kernel run once per row (seq_len = position + 1);
* bad block ids: error bit set, no fault, the other sequences unaffected;
  run-to-run determinism.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_golden, prefill_fixture_inputs
from oracle import paged_attention_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2.0 ** -7  # one bf16 ulp at magnitude 1 (see test_decode_gpu.py)


def _tol(dt: torch.dtype):
    return (BF16_TOL, BF16_TOL) if dt == torch.bfloat16 else (2e-3, 2e-3)


def _t16(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(getattr(torch, dtype)).to(device)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _row_meta(q_start, q_lens, tables, device):
    """positions, slot_mapping and cu_q of the rows, sequence after sequence."""
    pos, slots, cu = [], [], []
    r = 0
    for i, (qs, ql) in enumerate(zip(q_start, q_lens)):
        cu.append(r)
        for t in range(ql):
            p = qs + t
            pos.append(p)
            slots.append(int(tables[i][p // 16]) * 16 + p % 16)
        r += ql
    as_t = lambda x: torch.tensor(x, dtype=torch.int32, device=device)  # noqa: E731
    return as_t(pos), as_t(slots), as_t(cu)


def _prefill(K, q, k, v, inv_freq, pool, bt, q_start, q_lens, device, q_rot_out=None):
    pos, slots, cu = _row_meta(q_start, q_lens, bt.tolist(), device)
    q_rot = K.rope_reshape_and_cache(q, k, v, pos, slots, inv_freq, pool,
                                     q_out=q_rot_out if q_rot_out is not None else q.clone())
    qs = torch.tensor(q_start, dtype=torch.int32, device=device)
    ql = torch.tensor(q_lens, dtype=torch.int32, device=device)
    out = K.paged_prefill_attention(q_rot, pool, bt, qs, ql, cu, max(q_lens))
    torch.cuda.synchronize()
    return out, q_rot


PREFILL_FIXTURES = ["prefill_c1.npz", "prefill_c2.npz", "prefill_mha.npz", "prefill_g16.npz"]


@pytest.mark.parametrize("name", PREFILL_FIXTURES)
def test_golden_prefill(cuda_device, name):
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    d = load_golden(name)
    dt = str(d["dtype"])
    dev = cuda_device
    qb, kb, vb, pool_bits = prefill_fixture_inputs(d)
    pool = _t16(pool_bits, dt, dev)
    q, k, v = (_t16(x, dt, dev) for x in (qb, kb, vb))
    bt = torch.from_numpy(d["block_tables"]).to(dev)
    q_start = [int(x) for x in d["q_start"]]
    q_lens = [int(x) for x in d["q_lens"]]
    inv = rope_inv_freq(int(d["D"]), float(d["theta"])).to(dev)
    assert K.error_word(dev) == 0
    out, _ = _prefill(K, q, k, v, inv, pool, bt, q_start, q_lens, dev)
    assert K.error_word(dev) == 0
    # Written K bit-exact (kernel 1), V copied.
    pos, slots, _ = _row_meta(q_start, q_lens, d["block_tables"].tolist(), "cpu")
    pb = _bits(pool)
    for r, s in enumerate(slots.tolist()):
        np.testing.assert_array_equal(pb[s // 16, 0, s % 16], d["written_k"][r])
        np.testing.assert_array_equal(pb[s // 16, 1, s % 16], vb[r])
    atol, rtol = _tol(getattr(torch, dt))
    got = O.bits_to_f32(_bits(out), dt)
    ref = O.bits_to_f32(d["attn_out"], dt)
    if dt == "bfloat16":
        # The reference rounds Q.K^T (|s| ~ 10, one bf16 ulp = 2^-4) and P to
        # bf16 before the P.V product, so where the terms of an output cancel
        # two bf16 implementations differ by up to ~two ulps at magnitude 1.
        # Bar: all within 2 x 2^-7, 99.9 % within 2^-7 (the fp32 comparison
        # below holds the kernel to 2^-7 everywhere).
        np.testing.assert_allclose(got, ref, atol=2 * atol, rtol=2 * rtol)
        close = np.abs(got - ref) <= atol + rtol * np.abs(ref)
        assert close.mean() >= 0.999, close.mean()
    else:
        np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol)


def _torch_ref(q_rot, pool, tables, q_start, q_lens, G, scale):
    """fp32 causal attention over each sequence's paged K/V (rows sequence-major)."""
    n_q, D = q_rot.shape[1], q_rot.shape[2]
    out = torch.zeros(q_rot.shape, dtype=torch.float32, device=q_rot.device)
    r = 0
    for i, (qs, ql) in enumerate(zip(q_start, q_lens)):
        if ql == 0:
            continue
        L = qs + ql
        nb = (L + 15) // 16
        ids = torch.as_tensor(tables[i][:nb], device=q_rot.device, dtype=torch.long)
        Kf = pool[ids, 0].reshape(-1, pool.shape[3], D)[:L].float().repeat_interleave(G, 1)
        Vf = pool[ids, 1].reshape(-1, pool.shape[3], D)[:L].float().repeat_interleave(G, 1)
        q = q_rot[r:r + ql].float()
        s = torch.einsum("thd,lhd->htl", q, Kf) * scale
        kpos = torch.arange(L, device=q.device)
        qpos = qs + torch.arange(ql, device=q.device)
        s = s.masked_fill(kpos[None, None, :] > qpos[None, :, None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[r:r + ql] = torch.einsum("htl,lhd->thd", p, Vf)
        r += ql
    return out


CASES = [
    # n_q, n_kv, D, dtype, [(q_start, q_len)], theta
    (32, 4, 64, torch.float16, [(0, 300), (1000, 257), (5, 1), (40, 0), (0, 17)], 1e4),
    (32, 8, 128, torch.bfloat16, [(0, 513), (64, 100)], 5e5),
    (32, 2, 128, torch.float16, [(0, 77), (300, 40)], 1e4),
    (4, 4, 64, torch.float16, [(0, 260), (129, 128)], 1e4),
    (16, 8, 128, torch.float16, [(17, 129), (0, 1)], 1e4),
    (64, 8, 128, torch.float16, [(0, 200), (2048, 33)], 1e4),
    # A CTA holds two 128-row Q tiles: here the first needs one 128-key tile
    # fewer than the second, and the last CTAs hold a single partial tile.
    (8, 8, 64, torch.float16, [(100, 300), (0, 129), (7, 128)], 1e4),
    (16, 8, 128, torch.bfloat16, [(250, 700), (0, 64)], 5e5),
]


def _random_case(n_q, n_kv, D, dt, seqs, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ctx = [qs + ql for qs, ql in seqs]
    pages = [max(1, (c + 15) // 16) for c in ctx]
    nblk = sum(pages) + 7
    perm = torch.randperm(nblk, generator=g).tolist()
    tables, off = [], 0
    for p in pages:
        tables.append(perm[off:off + p])
        off += p
    bt = torch.zeros((len(seqs), max(pages)), dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    rows = sum(ql for _, ql in seqs)
    pool = torch.randn((nblk, 2, 16, n_kv, D), generator=g).to(dt).to(device)
    q = torch.randn((rows, n_q, D), generator=g).to(dt).to(device)
    k = torch.randn((rows, n_kv, D), generator=g).to(dt).to(device)
    v = torch.randn((rows, n_kv, D), generator=g).to(dt).to(device)
    return pool, q, k, v, bt.to(device), tables


@pytest.mark.parametrize("case", range(len(CASES)))
def test_prefill_matches_fp32_reference(cuda_device, case):
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    n_q, n_kv, D, dt, seqs, theta = CASES[case]
    dev = cuda_device
    pool, q, k, v, bt, tables = _random_case(n_q, n_kv, D, dt, seqs, dev, seed=case)
    inv = rope_inv_freq(D, theta).to(dev)
    q_start = [s[0] for s in seqs]
    q_lens = [s[1] for s in seqs]
    out, q_rot = _prefill(K, q, k, v, inv, pool, bt, q_start, q_lens, dev)
    assert K.error_word(dev) == 0
    ref = _torch_ref(q_rot, pool, tables, q_start, q_lens, n_q // n_kv, 1.0 / math.sqrt(D))
    atol, rtol = _tol(dt)
    torch.testing.assert_close(out.float(), ref, atol=atol, rtol=rtol)
    # Same result as the decode kernel run once per row.
    rows = q_rot.shape[0]
    if rows:
        row_bt = torch.cat([bt[i:i + 1].expand(ql, -1) for i, (_, ql) in enumerate(seqs)
                            if ql]).contiguous()
        row_sl = torch.tensor([qs + t + 1 for qs, ql in seqs for t in range(ql)],
                              dtype=torch.int32, device=dev)
        dec = K.paged_decode_attention(q_rot.contiguous(), pool, row_bt, row_sl)
        torch.testing.assert_close(out.float(), dec.float(), atol=atol, rtol=rtol)
    # Deterministic run to run.
    qs_t = torch.tensor(q_start, dtype=torch.int32, device=dev)
    ql_t = torch.tensor(q_lens, dtype=torch.int32, device=dev)
    _, _, cu = _row_meta(q_start, q_lens, bt.tolist(), dev)
    again = K.paged_prefill_attention(q_rot, pool, bt, qs_t, ql_t, cu, max(q_lens))
    assert torch.equal(again, out)


def test_prefill_strided_q_rows(cuda_device):
    """q as a slice of a fused QKV buffer (row stride (n_q + 2 n_kv) * D)."""
    from vllm_mps_b200 import kernels as K

    dev = cuda_device
    n_q, n_kv, D = 32, 4, 64
    seqs = [(0, 70), (33, 20)]
    pool, q, k, v, bt, tables = _random_case(n_q, n_kv, D, torch.float16, seqs, dev, seed=11)
    rows = q.shape[0]
    qkv = torch.randn((rows, (n_q + 2 * n_kv) * D), device=dev).half()
    qkv[:, : n_q * D] = q.reshape(rows, -1)
    q_view = qkv[:, : n_q * D].view(rows, n_q, D)  # strided rows
    qs = torch.tensor([s[0] for s in seqs], dtype=torch.int32, device=dev)
    ql = torch.tensor([s[1] for s in seqs], dtype=torch.int32, device=dev)
    _, _, cu = _row_meta([s[0] for s in seqs], [s[1] for s in seqs], bt.tolist(), dev)
    a = K.paged_prefill_attention(q_view, pool, bt, qs, ql, cu, 70)
    b = K.paged_prefill_attention(q.contiguous(), pool, bt, qs, ql, cu, 70)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_prefill_bad_block_id_sets_error_and_spares_other_sequences(cuda_device):
    from vllm_mps_b200 import kernels as K

    dev = cuda_device
    n_q, n_kv, D = 32, 4, 64
    seqs = [(0, 40), (0, 40)]
    pool, q, k, v, bt, tables = _random_case(n_q, n_kv, D, torch.float16, seqs, dev, seed=5)
    qs = torch.tensor([0, 0], dtype=torch.int32, device=dev)
    ql = torch.tensor([40, 40], dtype=torch.int32, device=dev)
    cu = torch.tensor([0, 40], dtype=torch.int32, device=dev)
    good = K.paged_prefill_attention(q, pool, bt, qs, ql, cu, 40).clone()
    bad = bt.clone()
    bad[1, 1] = pool.shape[0] + 1000  # out of range
    assert K.error_word(dev) == 0
    out = K.paged_prefill_attention(q, pool, bad, qs, ql, cu, 40)
    torch.cuda.synchronize()
    assert K.error_word(dev) & 2
    assert torch.equal(out[:40], good[:40])
    assert torch.isfinite(out[40:].float()).all()


def test_prefill_rejects_bad_arguments(cuda_device):
    from vllm_mps_b200 import kernels as K

    dev = cuda_device
    pool = torch.zeros((4, 2, 16, 4, 64), dtype=torch.float16, device=dev)
    q = torch.zeros((3, 24, 64), dtype=torch.float16, device=dev)  # G = 6
    z = torch.zeros(1, dtype=torch.int32, device=dev)
    bt = torch.zeros((1, 1), dtype=torch.int32, device=dev)
    with pytest.raises(NotImplementedError):
        K.paged_prefill_attention(q, pool, bt, z, z + 3, z, 3)
