"""The CPU oracles against the reference's own outputs (tests/golden/).

``tests/golden/make_golden.py`` ran the reference (Nihar0071/vllm_mps, its
CPU fallback path) and stored inputs and outputs; these tests pin both
oracles -- the numpy restatement and the C restatement -- to them:
written K/V bit-exact, attention output within 2e-3 absolute + relative
(one bf16 ulp at magnitude 1 for bf16, see test_decode_gpu.py).
"""

import hashlib

import numpy as np
import pytest

from conftest import golden_pool_bits, load_golden, prefill_fixture_inputs
from oracle import c_oracle
from oracle import paged_attention_oracle as O

FIXTURES = ["attn_c1_small.npz", "attn_c1_edges.npz", "attn_c1_b1.npz", "attn_c2_small.npz",
            "attn_c3_small.npz", "attn_mha_small.npz", "attn_g2_small.npz"]


def _inv_freq(d):
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    return rope_inv_freq(int(d["D"]), float(d["theta"])).numpy()


def _tol(dt):
    return (2.0 ** -7, 2.0 ** -7) if dt == "bfloat16" else (2e-3, 2e-3)


@pytest.mark.parametrize("name", FIXTURES)
def test_pool_regeneration_matches_reference(name):
    d = load_golden(name)
    bits = golden_pool_bits(d)
    assert hashlib.sha256(bits.tobytes()).hexdigest() == str(d["pool_sha256"])


@pytest.mark.parametrize("impl", ["numpy", "c"])
@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_reference(name, impl):
    d = load_golden(name)
    dt = str(d["dtype"])
    pool = golden_pool_bits(d)
    step = O.decode_step if impl == "numpy" else c_oracle.decode_step
    out, _ = step(d["q"], d["k"], d["v"], d["positions"], d["seq_lens"], d["block_tables"],
                  pool, _inv_freq(d), dt)
    sb, so = d["slot_block"], d["slot_off"]
    for i in range(len(sb)):
        np.testing.assert_array_equal(pool[sb[i], 0, so[i]], d["written_k"][i])
        np.testing.assert_array_equal(pool[sb[i], 1, so[i]], d["written_v"][i])
    atol, rtol = _tol(dt)
    got, ref = O.bits_to_f32(out, dt), O.bits_to_f32(d["attn_out"], dt)
    np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol)
    # The restatements follow the reference's rounding points, so nearly all
    # outputs are bit-identical (the rest differ in GEMM summation order).
    assert (out == d["attn_out"]).mean() > 0.9


def test_rope_tables_match_reference():
    for name in FIXTURES:
        d = load_golden(name)
        dt = str(d["dtype"])
        cos, sin = O.rope_cos_sin(d["positions"], _inv_freq(d))
        np.testing.assert_array_equal(O.round16(cos, dt), O.round16(d["cos_at_pos"], dt))
        np.testing.assert_array_equal(O.round16(sin, dt), O.round16(d["sin_at_pos"], dt))


def test_inv_freq_is_the_reference_expression():
    import torch
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    for D, th in ((64, 1e4), (128, 5e5)):
        ref = 1.0 / (th ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        assert torch.equal(rope_inv_freq(D, th), ref)


@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
def test_16bit_rounding_helpers(dt):
    import torch

    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 65504.0, 1e-8, -3e-5, 6.1e-5, 1e30], np.float32)])
    ref = torch.from_numpy(x).to(getattr(torch, dt)).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(O.f32_to_bits(x, dt), ref)


def test_oracle_bounds_checks_like_reference():
    pool = np.zeros((4, 2, 16, 1, 8), np.uint16)
    k = np.zeros((1, 1, 8), np.uint16)
    with pytest.raises(IndexError):
        O.write_kv(pool, [4], [0], k, k, 4, 16)
    with pytest.raises(IndexError):
        O.write_kv(pool, [0], [16], k, k, 4, 16)


def test_c_and_numpy_oracles_agree_on_a_ragged_batch():
    rng = np.random.default_rng(5)
    B, n_q, n_kv, D, nb = 6, 32, 4, 64, 128
    ctx = rng.integers(1, 300, size=B)
    pages = (ctx + 15) // 16
    perm = rng.permutation(nb)
    bt = np.zeros((B, pages.max()), np.int32)
    off = 0
    for i, p in enumerate(pages):
        bt[i, :p] = perm[off:off + p]
        off += p
    pool = O.f32_to_bits(rng.standard_normal((nb, 2, 16, n_kv, D), dtype=np.float32), "float16")
    q = O.f32_to_bits(rng.standard_normal((B, n_q, D), dtype=np.float32), "float16")
    k = O.f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), "float16")
    v = O.f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), "float16")
    inv = O.rope_inv_freq(D, 1e4)
    p1, p2 = pool.copy(), pool.copy()
    o1, _ = O.decode_step(q, k, v, ctx - 1, ctx, bt, p1, inv, "float16")
    o2, _ = c_oracle.decode_step(q, k, v, ctx - 1, ctx, bt, p2, inv, "float16")
    np.testing.assert_array_equal(p1, p2)
    np.testing.assert_allclose(O.bits_to_f32(o1, "float16"), O.bits_to_f32(o2, "float16"),
                               atol=2e-3, rtol=2e-3)


PREFILL_FIXTURES = ["prefill_c1.npz", "prefill_c2.npz", "prefill_mha.npz", "prefill_g16.npz"]


@pytest.mark.parametrize("name", PREFILL_FIXTURES)
def test_prefill_oracle_matches_reference(name):
    d = load_golden(name)
    dt = str(d["dtype"])
    q, k, v, pool = prefill_fixture_inputs(d)
    assert hashlib.sha256(pool.tobytes()).hexdigest() == str(d["pool_sha256"])
    out, kr = O.prefill(q, k, v, d["q_start"], d["q_lens"], d["block_tables"], pool,
                        _inv_freq(d), dt)
    np.testing.assert_array_equal(kr, d["written_k"])
    atol, rtol = _tol(dt)
    np.testing.assert_allclose(O.bits_to_f32(out, dt), O.bits_to_f32(d["attn_out"], dt),
                               atol=atol, rtol=rtol)
    assert (out == d["attn_out"]).mean() > 0.9
