"""The pipelined engine loop and the kernel it rests on.

``kernels.embed_rmsnorm`` (each row's token from the host or from the last
step's device-side ids, its embedding row, the first RMSNorm) against an
embedding lookup followed by ``kernels.add_rmsnorm``: the same arithmetic in
the same order, so bit-identical.  ``LLMEngine(pipeline=True)`` against the
synchronous loop on the same requests: identical tokens, step counts and
finish flags, through preemption (recompute and swap), finishing sequences
freeing blocks while their last step is still in flight, sampled (not only
greedy) rows, and steps that fall back to the eager forward mid-run.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,hidden", [(1, 2048), (13, 256), (256, 4096)])
def test_embed_rmsnorm_is_lookup_then_rmsnorm(cuda_device, dtype, rows, hidden):
    from vllm_mps_b200 import kernels as K

    g = torch.Generator(device=cuda_device).manual_seed(rows + hidden)
    vocab = 1000
    table = torch.randn(vocab, hidden, generator=g, device=cuda_device).to(dtype)
    weight = (torch.rand(hidden, generator=g, device=cuda_device) + 0.5).to(dtype)
    tokens = torch.randint(0, vocab, (rows,), generator=g, device=cuda_device, dtype=torch.int32)
    prev = torch.randint(0, vocab, (rows + 7,), generator=g, device=cuda_device)
    src = torch.randint(-1, rows + 7, (rows,), generator=g, device=cuda_device, dtype=torch.int32)
    K.error_word(cuda_device)
    for use_src in (False, True):
        res, out = K.embed_rmsnorm(table, weight, 1e-5, tokens, src=src if use_src else None,
                                   prev=prev if use_src else None)
        tok = torch.where(src >= 0, prev[src.clamp(min=0).long()], tokens.long()) if use_src \
            else tokens.long()
        want_res = table[tok]
        want = K.add_rmsnorm(want_res.clone(), weight, 1e-5)
        assert torch.equal(res.view(torch.int16), want_res.view(torch.int16))
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    assert K.error_word(cuda_device) == 0


def test_embed_rmsnorm_out_of_range_rows_are_flagged_and_zeroed(cuda_device):
    from vllm_mps_b200 import kernels as K

    table = torch.randn(50, 64, device=cuda_device, dtype=torch.float16)
    weight = torch.ones(64, device=cuda_device, dtype=torch.float16)
    tokens = torch.tensor([3, 50, 7, -2], device=cuda_device, dtype=torch.int32)
    prev = torch.tensor([11, 12], device=cuda_device)
    src = torch.tensor([-1, -1, 2, 1], device=cuda_device, dtype=torch.int32)
    K.error_word(cuda_device)
    res, out = K.embed_rmsnorm(table, weight, 1e-5, tokens, src=src, prev=prev)
    torch.cuda.synchronize(cuda_device)
    assert K.error_word(cuda_device) & 128
    # Row 0: token 3; row 1: 50 >= vocab; row 2: src 2 >= len(prev); row 3: prev[1] = 12.
    assert torch.equal(res[0], table[3]) and torch.equal(res[3], table[12])
    assert not res[1].any() and not res[2].any() and not out[1].any() and not out[2].any()
    with pytest.raises(ValueError):
        K.embed_rmsnorm(table, weight, 1e-5, tokens, src=src)  # src without prev


def _model(seed=3):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=1024,
                      rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096,
                      tie_word_embeddings=False)
    torch.manual_seed(seed)
    return LlamaForCausalLM(cfg).to(torch.float16).eval().cuda()


def _run(pipeline, blocks, swap, sampled=False, eager_every=0, seed=21):
    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.engine.llm_engine import LLMEngine

    # The 50 % watermark keeps 8 of 16 blocks in reserve, enough for the 8
    # sequences of a full batch to each open a block in one step, so a small
    # pool preempts instead of running out (the reference rule can).
    eng = LLMEngine.from_model(_model(), num_gpu_blocks=blocks, num_cpu_blocks=64,
                               max_batch_size=8, max_tokens_per_step=10 ** 6, mode="physical",
                               swap=swap, device="cuda", pipeline=pipeline,
                               preempt_watermark=0.5)
    if eager_every:
        real = eng._graphs.can_run
        asked = [0]

        def can_run(seq_ids):
            asked[0] += 1
            return real(seq_ids) and asked[0] % eager_every != 0

        eng._graphs.can_run = can_run
    swaps = [0]
    real_out = eng.kv_cache_manager.swap_out

    def swap_out(seq_id):
        swaps[0] += 1
        return real_out(seq_id)

    eng.kv_cache_manager.swap_out = swap_out
    rng = np.random.default_rng(seed)
    reqs = []
    for i in range(10):
        prompt = rng.integers(0, 1024, size=int(rng.integers(5, 60))).tolist()
        sp = SamplingParams(temperature=0.8 if sampled and i % 2 else 0.0, top_k=40,
                            max_tokens=int(rng.integers(3, 40)))
        reqs.append(eng.add_request(prompt, sp))
    torch.manual_seed(1234)  # the sampled rows' random stream
    calls, returned = 0, []
    while not eng.is_finished():
        returned += [(o.request_id, o.token_ids[-1], o.finished) for o in eng.step()]
        calls += 1
        assert calls < 1000
    outs = {r: (list(eng.get_output(r).token_ids), eng.get_output(r).finished,
                eng.get_output(r).num_steps) for r in reqs}
    return outs, returned, eng.total_tokens_generated, eng, swaps[0]


@pytest.mark.parametrize("swap", [False, True])
@pytest.mark.parametrize("blocks", [400, 16])
def test_pipelined_engine_matches_synchronous_engine(blocks, swap):
    """16 blocks (8 usable) for 10 requests of up to ~100 tokens force preemption."""
    sync, ret_s, n_s, _, pre_s = _run(False, blocks, swap)
    pipe, ret_p, n_p, eng, pre_p = _run(True, blocks, swap)
    assert pre_p == pre_s and (pre_s > 0) == (blocks == 16)
    assert pipe == sync
    assert n_p == n_s == sum(len(t) for t, _, _ in sync.values())
    # Every generated token is returned exactly once, in the same order.
    assert ret_p == ret_s
    assert all(fin for _, fin, _ in pipe.values())
    assert eng._inflight is None
    for s in eng._seqs.values():
        assert -1 not in s.token_ids  # every placeholder was resolved


def test_pipelined_engine_sampled_rows_and_eager_fallback():
    sync, ret_s, _, _, _ = _run(False, 16, False, sampled=True, eager_every=4)
    pipe, ret_p, _, _, _ = _run(True, 16, False, sampled=True, eager_every=4)
    assert pipe == sync and ret_p == ret_s


def test_pipelined_generate_and_is_finished():
    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.engine.llm_engine import LLMEngine

    eng = LLMEngine.from_model(_model(), num_gpu_blocks=64, num_cpu_blocks=8, max_batch_size=4,
                               mode="physical", device="cuda", pipeline=True)
    ids = eng.generate([5, 6, 7, 8], max_tokens=6, temperature=0.0)
    assert len(ids) == 6 and all(0 <= t < 1024 for t in ids)
    eng.add_request([9, 10], SamplingParams(temperature=0.0, max_tokens=1))
    assert not eng.is_finished()
    first = eng.step()  # launches the only step; nothing resolved yet
    assert first == [] and not eng.is_finished()  # its step is still in flight
    second = eng.step()
    assert len(second) == 1 and second[0].finished and eng.is_finished()
