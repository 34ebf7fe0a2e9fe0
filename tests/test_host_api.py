"""Host-side API that needs no GPU: the C-ABI library, the pool API, metadata, sampling.

* The shared library loads here (it links no libcuda) and exports every
  function ``include/vmps.h`` declares; host-side argument checks return
  the documented status codes before any CUDA call.
* The pool keeps the reference's layout, method set and ``IndexError``
  bounds checks (memory/mps_memory_pool.py:82-268; the reference's
  tests/test_memory_pool.py cases).
* Step metadata (block tables, slot mapping) matches the reference's
  addressing (models/llama_adapter.py:175-196).
* Greedy sampling picks the first index on ties (model/sampler.py:33-34).
"""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "vmps.h")


def _declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\*?(vmps_[a-z_0-9]+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from vllm_mps_b200 import kernels as K

    lib = K.load_library()
    declared = _declared_functions()
    assert "vmps_paged_decode_step" in declared and len(declared) >= 8
    for name in declared:
        assert hasattr(lib, name), name
    assert set(K.EXPORTED_SYMBOLS) <= set(declared)
    assert lib.vmps_version().startswith(b"vmps")


def test_host_side_argument_checks_need_no_gpu():
    from vllm_mps_b200 import kernels as K

    lib = K.load_library()
    # Bad dtype / sizes are rejected before any CUDA call.
    rc = lib.vmps_rope_reshape_and_cache(None, None, 0, None, 0, None, 0, None, None, None, None,
                                         4, 8, 2, 64, 16, 10, 7, None)
    assert rc == -1 and b"dtype" in lib.vmps_last_error()
    rc = lib.vmps_paged_decode_attention(None, None, None, None, 1, None, 4, 8, 2, 96, 16, 10,
                                         0.1, None, 0, 0, None)
    assert rc == -2  # head_dim 96 not built
    rc = lib.vmps_paged_decode_attention(None, None, None, None, 1, None, 4, 8, 2, 64, 32, 10,
                                         0.1, None, 0, 0, None)
    assert rc == -2 and b"block_size" in lib.vmps_last_error()
    rc = lib.vmps_paged_decode_attention(None, None, None, None, 1, None, 0, 8, 2, 64, 16, 10,
                                         0.1, None, 0, 0, None)
    assert rc == 0  # empty batch: nothing to do
    # Misaligned pointers are refused on the host (the kernels are never
    # given an address their 16-byte loads or 16-bit stores cannot use).
    # The pointers are never dereferenced on this path.
    base = 1 << 20
    rc = lib.vmps_paged_decode_attention(base, base + 8, base, base, 1, base, 4, 8, 2, 64, 16, 10,
                                         0.1, None, 0, 0, None)
    assert rc == -3 and b"aligned" in lib.vmps_last_error()  # q not 16-byte aligned
    rc = lib.vmps_paged_decode_attention(base + 1, base, base, base, 1, base, 4, 8, 2, 64, 16, 10,
                                         0.1, None, 0, 0, None)
    assert rc == -3 and b"out must be 2-byte aligned" in lib.vmps_last_error()
    # Decode GEMM: shapes outside what is built are refused before any CUDA call.
    assert lib.vmps_decode_gemm_supported(8, 2560, 2048, 0) == 1
    assert lib.vmps_decode_gemm_supported(9, 2560, 2048, 0) == 0   # M <= 8
    assert lib.vmps_decode_gemm_supported(8, 2564, 2048, 0) == 0   # N % 8
    assert lib.vmps_decode_gemm_supported(8, 2560, 2080, 0) == 0   # K % 64
    assert lib.vmps_decode_gemm_supported(8, 2560, 16384, 0) == 0  # K <= 8192
    rc = lib.vmps_decode_gemm(None, 0, None, 0, None, 9, 2560, 2048, 0, 0, None)
    assert rc == -2 and b"M=9" in lib.vmps_last_error()
    rc = lib.vmps_add_rmsnorm(None, 0, None, 0, None, 0, None, 4, 12, 1e-5, 0, None)
    assert rc == -1 and b"hidden=12" in lib.vmps_last_error()


def test_kernel_wrappers_refuse_cpu_tensors():
    from vllm_mps_b200 import kernels as K

    pool = torch.zeros(4, 2, 16, 2, 64, dtype=torch.float16)
    q = torch.zeros(1, 4, 64, dtype=torch.float16)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    sl = torch.ones(1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        K.paged_decode_attention(q, pool, bt, sl)


def test_pool_layout_and_reference_api_on_host():
    from vllm_mps_b200.memory.mps_memory_pool import MPSMemoryPool

    pool = MPSMemoryPool(8, 4, 2, 8, dtype=torch.float32, device="cpu")
    assert list(pool._pool.shape) == [8, 2, 4, 2, 8]
    k, v = torch.randn(2, 8), torch.randn(2, 8)
    pool.write_kv(1, 3, k, v)
    k1, v1 = pool.read_kv(1, 3)
    assert torch.equal(k1, k) and torch.equal(v1, v)
    for bid in (0, 1):
        for pos in range(4):
            pool.write_kv(bid, pos, torch.full((2, 8), float(bid * 4 + pos)),
                          torch.full((2, 8), float(bid * 4 + pos + 100)))
    kk, vv = pool.gather_blocks([0, 1])
    assert kk.shape == (8, 2, 8) and torch.equal(kk[:, 0, 0], torch.arange(8.0))
    assert torch.equal(vv[:, 1, 3], torch.arange(8.0) + 100)
    pool.copy_block(0, 5)
    assert torch.equal(pool.read_block_kv(5)[0], pool.read_block_kv(0)[0])
    with pytest.raises(IndexError):
        pool.write_kv(8, 0, k, v)
    with pytest.raises(IndexError):
        pool.write_kv(0, 4, k, v)
    with pytest.raises(IndexError):
        pool.copy_block(0, -1)
    assert pool.get_memory_mb() > 0


def test_per_layer_pool_and_swap_space_on_host():
    from vllm_mps_b200.memory.cuda_memory_pool import CUDAMemoryPool, SwapSpace

    pool = CUDAMemoryPool(6, 16, 2, 64, torch.float16, "cpu", num_layers=3)
    assert pool.layer(2).shape == (6, 2, 16, 2, 64)
    pool.layer(1)[2].fill_(3.0)
    pool.layer(2)[2].fill_(5.0)
    swap = SwapSpace(pool, 4)
    swap.copy_out([2], [1])
    pool._all.zero_()
    swap.copy_in([1], [4])
    assert float(pool.layer(1)[4].float().mean()) == 3.0
    assert float(pool.layer(2)[4].float().mean()) == 5.0
    pool.copy_block(4, 0)
    assert float(pool.layer(2)[0].float().mean()) == 5.0


def test_step_metadata_matches_reference_addressing():
    from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
    from vllm_mps_b200.models.llama_adapter import build_step_metadata

    kv = KVCacheManager(32, 4)
    lens = [1, 16, 17, 40]
    for sid, n in enumerate(lens):
        kv.allocate(sid)
        for _ in range(n):
            kv.append_slot(sid)
    meta = build_step_metadata(kv, list(range(4)), [n - 1 for n in lens], lens, 16,
                               torch.device("cpu"))
    tables = [kv.get_block_table(s) for s in range(4)]
    assert meta.bt_tensor.shape == (4, 3)
    for i, t in enumerate(tables):
        assert meta.bt_tensor[i, :len(t)].tolist() == t
        assert meta.bt_tensor[i, len(t):].eq(0).all()
        p = lens[i] - 1
        assert int(meta.slot_mapping[i]) == t[p // 16] * 16 + p % 16
        assert meta.write_info[i].tolist() == [t[p // 16], p % 16]
    assert meta.sl_tensor.tolist() == lens and meta.pos_tensor.tolist() == [n - 1 for n in lens]


def test_prefill_metadata_rows_and_sequences():
    from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
    from vllm_mps_b200.models.llama_adapter import build_prefill_metadata

    kv = KVCacheManager(32, 4)
    lens = [5, 40, 17]
    for sid, n in enumerate(lens):
        kv.allocate(sid)
        for _ in range(n):
            kv.append_slot(sid)
    pieces = [(0, 0, 4), (1, 16, 23), (2, 0, 16)]  # sequence 1 resumes at position 16
    meta = build_prefill_metadata(kv, pieces, 16, torch.device("cpu"))
    tables = [kv.get_block_table(s) for s in range(3)]
    assert meta.rows == 43 and meta.max_q_len == 23
    assert meta.q_start.tolist() == [0, 16, 0] and meta.q_lens.tolist() == [4, 23, 16]
    assert meta.cu_q.tolist() == [0, 4, 27]
    for i, t in enumerate(tables):
        assert meta.bt_tensor[i, :len(t)].tolist() == t
    r = 0
    for sid, qs, ql in pieces:
        for p in range(qs, qs + ql):
            assert int(meta.pos_tensor[r]) == p
            assert int(meta.slot_mapping[r]) == tables[sid][p // 16] * 16 + p % 16
            r += 1


def test_greedy_sampler_takes_first_index_on_ties():
    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.model.sampler import Sampler

    logits = torch.tensor([[0.0, 3.0, 3.0, 1.0], [5.0, 5.0, 5.0, 5.0]])
    greedy = SamplingParams(temperature=0.0)
    assert Sampler().sample_rows(logits, [greedy, greedy]) == [1, 0]
    assert Sampler().sample(logits[0], greedy) == 1
    g = torch.Generator().manual_seed(0)
    tok = Sampler().sample_rows(logits, [SamplingParams(temperature=1.0, top_k=1), greedy], g)
    # top-k keeps every logit >= the k-th largest (model/sampler.py:37-41): both 3.0s.
    assert tok[0] in (1, 2) and tok[1] == 0


def test_batched_sampling_matches_reference_distribution():
    """Temperature + top-k + top-p of several rows in one batched pass give
    each row the distribution of the reference's per-row steps
    (model/sampler.py:36-59): same support, frequencies within sampling noise."""
    import torch.nn.functional as F

    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.model.sampler import Sampler

    torch.manual_seed(0)
    logits = torch.randn(4, 50)
    params = [SamplingParams(temperature=0.7, top_k=5), SamplingParams(temperature=1.3, top_p=0.6),
              SamplingParams(temperature=1.0, top_k=10, top_p=0.8), SamplingParams(temperature=0.0)]

    def reference_probs(l, p):
        l = l / p.temperature
        if p.top_k > 0:
            th = torch.topk(l, p.top_k).values[-1]
            l = torch.where(l < th, torch.tensor(float("-inf")), l)
        if p.top_p < 1.0:
            sl, si = torch.sort(l, descending=True)
            pr = F.softmax(sl, -1)
            sl = sl.masked_fill(torch.cumsum(pr, -1) - pr >= p.top_p, float("-inf"))
            l = torch.zeros_like(l).scatter_(-1, si, sl)
        return F.softmax(l, -1)

    g = torch.Generator().manual_seed(1)
    counts = torch.zeros(4, 50)
    n = 3000
    for _ in range(n):
        for r, t in enumerate(Sampler().sample_rows(logits, params, g)):
            counts[r, t] += 1
    for r in range(3):
        ref = reference_probs(logits[r], params[r])
        emp = counts[r] / n
        assert torch.equal(emp > 0, ref > 0), r
        assert (emp - ref).abs().max() < 0.03, r
    assert counts[3, int(torch.argmax(logits[3]))] == n


def test_model_config_from_hf_config():
    from transformers import LlamaConfig

    from vllm_mps_b200.core.model_config import ModelConfig

    hf = LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8,
                     num_hidden_layers=32, vocab_size=128256, rope_theta=500000.0,
                     max_position_embeddings=8192)
    cfg = ModelConfig.from_hf_config(hf, "llama3-shape", device="cpu")
    assert (cfg.n_heads, cfg.n_kv_heads, cfg.d_k, cfg.architecture) == (32, 8, 128, "llama")
    assert cfg.rope_theta == 500000.0 and cfg.get_kv_cache_config()["n_heads"] == 8


def test_decode_graph_buckets():
    """Batch sizes map to the smallest bucket that holds them; larger batches run eagerly."""
    from vllm_mps_b200.engine.decode_graph import BUCKETS, DecodeGraphRunner

    assert [DecodeGraphRunner.bucket(b) for b in (1, 2, 3, 8, 9, 256, 257, 512)] == \
        [1, 2, 4, 8, 16, 256, 512, 512]
    assert DecodeGraphRunner.bucket(BUCKETS[-1] + 1) is None
    assert list(BUCKETS) == sorted(BUCKETS)


def test_decode_graph_fused_layer_eligibility():
    """A stock HF Llama takes the fused element-wise path (its SiLU is transformers'
    own activation class); a model whose MLP is not SiLU-gated replays HF modules."""
    from types import SimpleNamespace

    import torch.nn as nn
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_mps_b200.engine.decode_graph import DecodeGraphRunner

    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=100)
    model = LlamaForCausalLM(cfg).eval()
    r = DecodeGraphRunner.__new__(DecodeGraphRunner)
    r.adapter = SimpleNamespace(hf_model=model, model_config=SimpleNamespace(d_model=64))
    assert r._llama_layers()
    w_gate = model.model.layers[1].mlp.gate_proj.weight.detach().clone()
    fused = r._fuse_gate_up()
    assert fused[1].shape == (256, 64) and torch.equal(fused[1][:128], w_gate)
    # The module weights are views of the fused buffer: one copy of the weights.
    assert model.model.layers[1].mlp.up_proj.weight.data_ptr() == fused[1][128:].data_ptr()
    # Kernels a replayed step launches: at decode batch sizes every projection
    # is a decode GEMM (SiLU * up fused), so 7 per layer plus the first norm
    # and the LM head; here the 100-row vocabulary is not a multiple of 8, so
    # the LM head stays on cuBLAS.
    r._gate_up = fused
    a0 = model.model.layers[0].self_attn
    a0._w_qkv = torch.zeros(128, 64)
    a0.W_O = nn.Linear(64, 64, bias=False)
    model.model.layers[1].self_attn._w_qkv = a0._w_qkv
    model.model.layers[1].self_attn.W_O = a0.W_O
    r.adapter.model_config.d_model = 64
    assert r.own_kernels_per_step(8) == 7 * 2 + 1
    model.model.layers[0].mlp.act_fn = nn.GELU()
    assert not r._llama_layers()


def test_model_config_from_a_local_checkpoint_directory(tmp_path):
    """from_pretrained reads a saved config (no network): the way a user points the
    engine at a local model (core/model_config.py:50-96 of the reference)."""
    from transformers import LlamaConfig

    from vllm_mps_b200.core.model_config import ModelConfig

    LlamaConfig(hidden_size=256, num_attention_heads=8, num_key_value_heads=2,
                num_hidden_layers=3, vocab_size=1000, rope_theta=250000.0,
                max_position_embeddings=4096, architectures=["LlamaForCausalLM"]).save_pretrained(tmp_path)
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    assert (cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.d_k, cfg.n_layers) == (256, 8, 2, 32, 3)
    assert cfg.architecture == "llama" and cfg.rope_theta == 250000.0 and cfg.max_seq_len == 4096


def test_bench_tensor_peak_matches_the_timed_region(tmp_path, monkeypatch):
    """bench.py's tensor roofline uses the measured burst bf16 peak for a
    short timed region and the measured sustained one for a region of half a
    second or more (which runs under the power cap like the sustained loop),
    and reports the other figure beside it."""
    import json
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    (tmp_path / "MEASURED_PEAKS.json").write_text(
        json.dumps({"bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}))
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    peak, kind, other = bench.tensor_peak(0.05)
    assert peak == 1600.0 and kind.startswith("measured (burst") and other == (1400.0, "sustained")
    peak, kind, other = bench.tensor_peak(bench.SUSTAINED_AFTER_S)
    assert peak == 1400.0 and kind.startswith("measured (sustained") and other == (1600.0, "burst")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"bf16_tflops": 1600.0}))
    assert bench.tensor_peak(2.0)[:2] == (1600.0, "measured (burst: 2.000 s timed)")
    (tmp_path / "MEASURED_PEAKS.json").unlink()
    assert bench.tensor_peak(2.0) == (1590.0, "fallback", None)


def test_bench_algorithmic_bytes_of_config_1():
    """The roofline numerator bench.py reports for config 1, recomputed from
    its definition on the bench's seeded workload (rank 0): every context's
    K and V rows of all kv heads, q in and out, the block-table entries read
    and the lengths; the fused step adds the new token's k and v read, its
    rotated K and V written, and positions and slots read."""
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    cfg = bench.CONFIGS["c1"]
    B, n_q, n_kv, D = cfg[0], cfg[1], cfg[2], cfg[3]
    ctx, pages, _ = bench.make_host_workload(cfg, seed=1000)
    assert int(ctx.sum()) == 65186 and (pages == (ctx + 15) // 16).all()
    e = 2
    attn = (int(ctx.sum()) * n_kv * D * 2 * e + 2 * B * n_q * D * e
            + int(pages.sum()) * 4 + 4 * B)
    fused = attn + 2 * B * n_kv * D * e * 2 + 2 * 4 * B
    assert bench.alg_bytes(cfg, ctx, pages) == attn == 67291428
    assert bench.alg_bytes(cfg, ctx, pages, fused=True) == fused == 67423012


def test_bench_prefill_flops_count_causal_pairs():
    """The tensor roofline's numerator for kernel 3: 4 * n_q * D FLOPs (QK^T
    and PV, a multiply-add each) per causal (row, key) pair, L (L + 1) / 2
    pairs per prompt of L tokens."""
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    B, L, n_q, D = 16, 2048, 32, 128
    assert bench.prefill_flops(B, L, n_q, D) == B * L * (L + 1) // 2 * 4 * n_q * D == 550024249344
