"""Parity of the CUDA decode step (kernels 1 and 2) through the C ABI.

Checks, on a B200:
* against the reference's own outputs (``tests/golden/attn_*.npz``, made by
  running the reference's CPU path): written K/V bit-exact, attention output
  within 2e-3 absolute + relative (the bar of the spec; fp16/bf16 I/O with
  fp32 accumulation);
* against the CPU oracle on seeded cases the fixtures do not cover (G=16,
  bf16 with G=8, random ragged batches);
* at the full sizes of the benchmark configs (C1: 64 x U[1,2048] over a
  16384-block pool; C3: 4 x 131072 over 32768+ blocks) against a PyTorch
  fp32 reference evaluated on the GPU;
* edge cases: length-1 sequences, block boundaries, empty sequences, bad
  block ids and too-short block tables (error word set, no fault), merge
  counters back at zero, run-to-run determinism.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import golden_pool_bits, load_golden
from oracle import paged_attention_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3
# bf16 carries 8 significant bits: one ulp is 2^-7 relative, so 2e-3 is below
# a single rounding step for |x| > 0.25.  The reference also rounds scores and
# probabilities to bf16 before the P.V product, so bf16 outputs are held to
# one bf16 ulp at magnitude 1 (2^-7) absolute + relative instead.
BF16_TOL = 2.0 ** -7


def _tol(dtype: str):
    return (BF16_TOL, BF16_TOL) if dtype == "bfloat16" else (ATOL, RTOL)

ATTN_FIXTURES = [
    "attn_c1_small.npz", "attn_c1_edges.npz", "attn_c1_b1.npz", "attn_c2_small.npz",
    "attn_c3_small.npz", "attn_mha_small.npz", "attn_g2_small.npz",
]


def _t16(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(getattr(torch, dtype)).to(device)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _run_step(K, q, k, v, positions, slots, inv_freq, pool, block_tables, seq_lens):
    K.rope_reshape_and_cache(q, k, v, positions, slots, inv_freq, pool)
    out = K.paged_decode_attention(q, pool, block_tables, seq_lens)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_golden_decode_step(cuda_device, name):
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    d = load_golden(name)
    dt = str(d["dtype"])
    dev = cuda_device
    pool_bits = golden_pool_bits(d)
    pool = _t16(pool_bits, dt, dev)
    q = _t16(d["q"], dt, dev)
    k = _t16(d["k"], dt, dev)
    v = _t16(d["v"], dt, dev)
    bt = torch.from_numpy(d["block_tables"]).to(dev)
    sl = torch.from_numpy(d["seq_lens"]).to(dev)
    pos = torch.from_numpy(d["positions"]).to(dev)
    slots = torch.from_numpy((d["slot_block"].astype(np.int64) * int(d["block_size"])
                              + d["slot_off"]).astype(np.int32)).to(dev)
    inv = rope_inv_freq(int(d["D"]), float(d["theta"])).to(dev)
    out = _run_step(K, q, k, v, pos, slots, inv, pool, bt, sl)
    assert K.error_word(dev) == 0

    # Written K/V: bit-exact against the reference.
    pool_after = _bits(pool)
    sb, so = d["slot_block"], d["slot_off"]
    for i in range(len(sb)):
        np.testing.assert_array_equal(pool_after[sb[i], 0, so[i]], d["written_k"][i])
        np.testing.assert_array_equal(pool_after[sb[i], 1, so[i]], d["written_v"][i])
    # Every other slot untouched.
    expect = pool_bits.copy()
    for i in range(len(sb)):
        expect[sb[i], 0, so[i]] = d["written_k"][i]
        expect[sb[i], 1, so[i]] = d["written_v"][i]
    np.testing.assert_array_equal(pool_after, expect)
    # Q rotated in place = the reference's Q_rot.
    cos, sin = O.rope_cos_sin(d["positions"], inv.cpu().numpy())
    q_rot = O.apply_rope(O.bits_to_f32(d["q"], dt), cos, sin, dt)
    np.testing.assert_array_equal(_bits(q), O.f32_to_bits(q_rot, dt))
    # Attention output against the reference within 2e-3 abs + rel.
    got = O.bits_to_f32(_bits(out), dt)
    ref = O.bits_to_f32(d["attn_out"], dt)
    atol, rtol = _tol(dt)
    np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol)


def _seeded_case(seed, B, n_q, n_kv, D, dtype, ctx_lo, ctx_hi, num_blocks, device,
                 ctx=None, theta=10000.0, pool_on_device=False):
    rng = np.random.default_rng(seed)
    bs = 16
    if ctx is None:
        ctx = rng.integers(ctx_lo, ctx_hi + 1, size=B)
    ctx = np.asarray(ctx, dtype=np.int64)
    pages = (ctx + bs - 1) // bs
    assert pages.sum() <= num_blocks
    perm = rng.permutation(num_blocks)
    max_blocks = max(1, int(pages.max()))
    bt = np.zeros((B, max_blocks), dtype=np.int32)
    off = 0
    for i, p in enumerate(pages):
        bt[i, :p] = perm[off: off + p]
        off += p
    tdt = getattr(torch, dtype)
    g = torch.Generator(device="cpu").manual_seed(seed)
    if pool_on_device:
        gd = torch.Generator(device=device).manual_seed(seed)
        pool = torch.randn((num_blocks, 2, bs, n_kv, D), generator=gd, device=device,
                           dtype=torch.float32).to(tdt)
    else:
        pool = torch.randn((num_blocks, 2, bs, n_kv, D), generator=g).to(tdt)
    q = torch.randn((B, n_q, D), generator=g).to(tdt)
    k = torch.randn((B, n_kv, D), generator=g).to(tdt)
    v = torch.randn((B, n_kv, D), generator=g).to(tdt)
    pos = np.maximum(ctx - 1, 0)
    slot = np.array([bt[i, pos[i] // bs] * bs + pos[i] % bs for i in range(B)], dtype=np.int32)
    return dict(pool=pool.to(device), q=q.to(device), k=k.to(device), v=v.to(device),
                bt=torch.from_numpy(bt).to(device), sl=torch.from_numpy(ctx.astype(np.int32)).to(device),
                pos=torch.from_numpy(pos.astype(np.int32)).to(device),
                slot=torch.from_numpy(slot).to(device), ctx=ctx, bt_np=bt, dtype=dtype,
                theta=theta, D=D)


@pytest.mark.parametrize("cfg", [
    # seed, B, n_q, n_kv, D, dtype, lo, hi, blocks
    (101, 6, 64, 4, 64, "float16", 1, 400, 256),     # G = 16
    (102, 5, 64, 8, 128, "bfloat16", 1, 700, 320),   # G = 8, bf16
    (103, 7, 32, 8, 128, "float16", 1, 300, 256),    # G = 4 (Llama-3-8B heads)
    (104, 3, 4, 1, 128, "float16", 1, 500, 128),     # n_kv = 1
    (105, 9, 16, 16, 64, "bfloat16", 1, 200, 256),   # MHA, 16 kv heads
])
def test_oracle_decode_step(cuda_device, cfg):
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    seed, B, n_q, n_kv, D, dt, lo, hi, nb = cfg
    c = _seeded_case(seed, B, n_q, n_kv, D, dt, lo, hi, nb, cuda_device)
    pool_bits = _bits(c["pool"])
    q_bits, k_bits, v_bits = _bits(c["q"]), _bits(c["k"]), _bits(c["v"])
    inv = rope_inv_freq(D, c["theta"])
    out = _run_step(K, c["q"], c["k"], c["v"], c["pos"], c["slot"], inv.to(cuda_device),
                    c["pool"], c["bt"], c["sl"])
    assert K.error_word(cuda_device) == 0
    ref_out, _ = O.decode_step(q_bits, k_bits, v_bits, c["pos"].cpu().numpy(), c["ctx"],
                               c["bt_np"], pool_bits, inv.numpy(), dt)
    np.testing.assert_array_equal(_bits(c["pool"]), pool_bits)  # oracle wrote the same slots
    atol, rtol = _tol(dt)
    np.testing.assert_allclose(O.bits_to_f32(_bits(out), dt), O.bits_to_f32(ref_out, dt),
                               atol=atol, rtol=rtol)


def _torch_fp32_attention(q, pool, bt_np, ctx, block_size=16):
    """fp32 PyTorch reference on the GPU (for sizes the CPU oracle is too slow for)."""
    B, n_q, D = q.shape
    n_kv = pool.shape[3]
    G = n_q // n_kv
    out = torch.empty(B, n_q, D, dtype=torch.float32, device=q.device)
    for i in range(B):
        L = int(ctx[i])
        nb = (L + block_size - 1) // block_size
        ids = torch.from_numpy(bt_np[i, :nb].astype(np.int64)).to(q.device)
        kk = pool[ids, 0].reshape(-1, n_kv, D)[:L].float()  # (L, n_kv, D)
        vv = pool[ids, 1].reshape(-1, n_kv, D)[:L].float()
        qq = q[i].float().view(n_kv, G, D)  # query head h uses kv head h // G
        s = torch.einsum("kgd,lkd->kgl", qq, kk) / math.sqrt(D)
        out[i] = torch.einsum("kgl,lkd->kgd", torch.softmax(s, dim=-1), vv).reshape(n_q, D)
    return out


@pytest.mark.parametrize("which", ["c1", "c3"])
def test_full_size_configs(cuda_device, which):
    """Benchmark-size inputs against a GPU fp32 PyTorch reference (2e-3 abs+rel)."""
    from vllm_mps_b200 import kernels as K

    if which == "c1":
        c = _seeded_case(1, 64, 32, 4, 64, "float16", 1, 2048, 16384, cuda_device,
                         pool_on_device=True)
    else:
        c = _seeded_case(3, 4, 64, 8, 128, "float16", 0, 0, 32768 + 64, cuda_device,
                         ctx=[131072] * 4, pool_on_device=True)
    out = K.paged_decode_attention(c["q"], c["pool"], c["bt"], c["sl"])
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) == 0
    ref = _torch_fp32_attention(c["q"], c["pool"], c["bt_np"], c["ctx"])
    torch.testing.assert_close(out.float(), ref, atol=ATOL, rtol=RTOL)
    # Deterministic: a second run gives identical bits.
    out2 = K.paged_decode_attention(c["q"], c["pool"], c["bt"], c["sl"])
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))


def test_fused_step_matches_kernel1_then_kernel2(cuda_device):
    """The one-launch step == kernel 1 + kernel 2, bit for bit; q is left unrotated."""
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    for dt, n_q, n_kv, D in (("float16", 32, 4, 64), ("bfloat16", 32, 8, 128),
                             ("float16", 64, 4, 64)):
        c = _seeded_case(7, 8, n_q, n_kv, D, dt, 1, 2000, 2048, cuda_device)
        inv = rope_inv_freq(D, 10000.0).to(cuda_device)
        pool0, q0 = c["pool"].clone(), c["q"].clone()
        ref = _run_step(K, c["q"], c["k"], c["v"], c["pos"], c["slot"], inv, c["pool"], c["bt"],
                        c["sl"])
        q1, pool1 = q0.clone(), pool0.clone()
        for _ in range(2):  # twice: the merge counters must be back at zero
            out = K.paged_decode_step(q1, c["k"], c["v"], c["pos"], c["slot"], inv, pool1,
                                      c["bt"], c["sl"])
            torch.cuda.synchronize()
            assert K.error_word(cuda_device) == 0
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
            assert torch.equal(pool1.view(torch.int16), c["pool"].view(torch.int16))
            assert torch.equal(q1.view(torch.int16), q0.view(torch.int16))


def test_fused_step_strided_qkv_and_golden(cuda_device):
    """Fused step on slices of one packed QKV row (the fused-projection layout)."""
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    d = load_golden("attn_c3_small.npz")
    dt = str(d["dtype"])
    n_q, n_kv, D = int(d["n_q"]), int(d["n_kv"]), int(d["D"])
    B = d["q"].shape[0]
    pool = _t16(golden_pool_bits(d), dt, cuda_device)
    qkv = torch.empty(B, (n_q + 2 * n_kv) * D, dtype=getattr(torch, dt), device=cuda_device)
    qkv[:, : n_q * D] = _t16(d["q"], dt, cuda_device).reshape(B, -1)
    qkv[:, n_q * D: (n_q + n_kv) * D] = _t16(d["k"], dt, cuda_device).reshape(B, -1)
    qkv[:, (n_q + n_kv) * D:] = _t16(d["v"], dt, cuda_device).reshape(B, -1)
    q = qkv[:, : n_q * D].view(B, n_q, D)
    k = qkv[:, n_q * D: (n_q + n_kv) * D]
    v = qkv[:, (n_q + n_kv) * D:]
    slots = torch.from_numpy((d["slot_block"].astype(np.int64) * 16 + d["slot_off"])
                             .astype(np.int32)).to(cuda_device)
    out = K.paged_decode_step(q, k, v, torch.from_numpy(d["positions"]).to(cuda_device), slots,
                              rope_inv_freq(D, float(d["theta"])).to(cuda_device), pool,
                              torch.from_numpy(d["block_tables"]).to(cuda_device),
                              torch.from_numpy(d["seq_lens"]).to(cuda_device))
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) == 0
    pool_after = _bits(pool)
    for i in range(B):
        np.testing.assert_array_equal(pool_after[d["slot_block"][i], 0, d["slot_off"][i]], d["written_k"][i])
        np.testing.assert_array_equal(pool_after[d["slot_block"][i], 1, d["slot_off"][i]], d["written_v"][i])
    np.testing.assert_allclose(O.bits_to_f32(_bits(out), dt), O.bits_to_f32(d["attn_out"], dt),
                               atol=ATOL, rtol=RTOL)


def test_edge_lengths_and_empty(cuda_device):
    from vllm_mps_b200 import kernels as K

    ctx = [1, 0, 16, 17, 0, 33, 2047, 2048, 1]
    c = _seeded_case(9, len(ctx), 32, 4, 64, "float16", 0, 0, 1024, cuda_device, ctx=ctx)
    out = K.paged_decode_attention(c["q"], c["pool"], c["bt"], c["sl"])
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) == 0
    got = out.float().cpu()
    for i, L in enumerate(ctx):
        if L == 0:
            assert torch.count_nonzero(got[i]) == 0
    nz = [i for i, L in enumerate(ctx) if L > 0]
    ref = _torch_fp32_attention(c["q"][nz], c["pool"], c["bt_np"][nz], np.array(ctx)[nz])
    torch.testing.assert_close(out[nz].float(), ref, atol=ATOL, rtol=RTOL)
    # ctx = 1 attends to exactly its own (single) slot: output = that V row.
    v_first = c["pool"][int(c["bt_np"][0, 0]), 1, 0]  # (n_kv, D)
    torch.testing.assert_close(out[0].view(4, 8, 64).float(),
                               v_first.float().unsqueeze(1).expand(4, 8, 64), atol=1e-3, rtol=0)


def test_bad_block_ids_flag_without_fault(cuda_device):
    from vllm_mps_b200 import kernels as K

    c = _seeded_case(11, 4, 32, 4, 64, "float16", 40, 90, 64, cuda_device)
    bt = c["bt"].clone()
    bt[1, 0] = 10_000_000   # beyond the pool
    bt[2, 1] = -5
    K.error_word(cuda_device)
    K.paged_decode_attention(c["q"], c["pool"], bt, c["sl"])
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) & 2
    # Too-short block table: seq_len beyond max_blocks * 16.
    sl = c["sl"].clone()
    sl[0] = 16 * bt.shape[1] + 5
    K.paged_decode_attention(c["q"], c["pool"], c["bt"], sl)
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) & 4
    # Slot beyond the pool in kernel 1: skipped and flagged, nothing else moves.
    slot = c["slot"].clone()
    slot[0] = 64 * 16 + 3
    before = c["pool"].clone()
    K.rope_reshape_and_cache(c["q"], c["k"], c["v"], c["pos"], slot, None, c["pool"])
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) & 1
    changed = (before.view(torch.int16) != c["pool"].view(torch.int16)).any(dim=-1).any(dim=-1)
    blocks, kinds, offs = torch.nonzero(changed, as_tuple=True)
    s_np = c["slot"].cpu().numpy()
    allowed = {(int(s_np[i]) // 16, int(s_np[i]) % 16) for i in range(1, 4)}
    assert {(int(b), int(o)) for b, o in zip(blocks, offs)} <= allowed


def test_fused_attention_reference_api(cuda_device):
    """kernels.fused_attention == the reference's fused_attention_metal_fast contract."""
    from vllm_mps_b200 import kernels as K

    d = load_golden("attn_c1_small.npz")
    dt = str(d["dtype"])
    pool = _t16(golden_pool_bits(d), dt, cuda_device)
    # The fused entry point takes already-rotated K; use the reference's written K.
    new_k = _t16(d["written_k"], dt, cuda_device)
    new_v = _t16(d["written_v"], dt, cuda_device)
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq
    cos, sin = O.rope_cos_sin(d["positions"], rope_inv_freq(int(d["D"]), float(d["theta"])).numpy())
    q_rot = O.f32_to_bits(O.apply_rope(O.bits_to_f32(d["q"], dt), cos, sin, dt), dt)
    queries = _t16(q_rot, dt, cuda_device).contiguous()
    write_info = torch.from_numpy(np.stack([d["slot_block"], d["slot_off"]], 1).astype(np.int32)).to(cuda_device)
    out = K.fused_attention_metal_fast(
        pool, new_k, new_v, queries, torch.from_numpy(d["block_tables"]).to(cuda_device),
        torch.from_numpy(d["seq_lens"]).to(cuda_device), write_info, 32, 4, 64, 16)
    torch.cuda.synchronize()
    np.testing.assert_allclose(O.bits_to_f32(_bits(out), dt), O.bits_to_f32(d["attn_out"], dt),
                               atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("shape", [
    # name, n_q, n_kv, D, dtype, context lengths
    ("one long among many one-page", 32, 4, 64, "float16", [4000] + [5] * 200),
    ("mostly empty (a padded graph bucket)", 32, 4, 64, "float16",
     [0] * 150 + [700, 1, 1300] + [0] * 100 + [64]),
    ("4096 tiny sequences", 32, 4, 64, "float16", [1 + (i * 7) % 16 for i in range(4096)]),
    ("G=16, head_dim 128, ragged", 64, 4, 128, "bfloat16", [(i * 977) % 3000 + 1 for i in range(40)]),
    ("64 kv heads (the supported maximum), MHA", 64, 64, 64, "float16",
     [(i * 311) % 900 + 1 for i in range(24)]),
])
def test_work_split_extremes(cuda_device, shape):
    """The cost-weighted split over pages and sequence starts at its extremes:
    outputs against fp32 attention, merge counters left at zero (a second
    call on the same workspace gives identical bits), no error bits."""
    from vllm_mps_b200 import kernels as K

    name, n_q, n_kv, D, dt, ctx = shape
    pages = sum((c + 15) // 16 for c in ctx)
    c = _seeded_case(77, len(ctx), n_q, n_kv, D, dt, 0, 0, pages + 64, cuda_device, ctx=ctx,
                     pool_on_device=True)
    ws = K.DecodeWorkspace()
    out = K.paged_decode_attention(c["q"], c["pool"], c["bt"], c["sl"], workspace=ws)
    out2 = K.paged_decode_attention(c["q"], c["pool"], c["bt"], c["sl"], workspace=ws)
    torch.cuda.synchronize()
    assert K.error_word(cuda_device) == 0, name
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16)), name
    nz = [i for i, L in enumerate(ctx) if L > 0]
    z = [i for i, L in enumerate(ctx) if L == 0]
    if z:
        assert torch.count_nonzero(out[z]) == 0
    ref = _torch_fp32_attention(c["q"][nz], c["pool"], c["bt_np"][nz], np.array(ctx)[nz])
    atol, rtol = _tol(dt)
    torch.testing.assert_close(out[nz].float(), ref, atol=atol, rtol=rtol)
