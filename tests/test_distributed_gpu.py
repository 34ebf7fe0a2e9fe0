"""Sequence-sharded engine over NCCL: one process per GPU (up to 2 here).

Each rank runs a physical-mode engine with its own pool and allocator on its
own GPU; sampled tokens are gathered with one NCCL all-gather per step.  The
assembled tokens must equal an unsharded single-engine run, up to the first
decision whose top-1/top-2 logit margin in the unsharded run is below 0.05
(the non-attention GEMMs may pick different kernels for different batch
sizes, which can flip a near tie).  With one GPU the test runs a world of
one rank, which still goes through NCCL.
"""

import datetime
import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu


def _small_llama(seed=3):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=512, intermediate_size=2048, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=1024,
                      rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096,
                      tie_word_embeddings=False)
    torch.manual_seed(seed)
    return LlamaForCausalLM(cfg).to(torch.float16).eval()


def _workload():
    import numpy as np

    from vllm_mps_b200.core.sequence import SamplingParams

    rng = np.random.default_rng(5)
    lens = [3, 40, 17, 64, 1, 29, 90, 8, 33]
    prompts = [rng.integers(0, 1024, size=n).tolist() for n in lens]
    params = [SamplingParams(temperature=0.0, max_tokens=4 + (3 * i) % 11) for i in range(len(lens))]
    return prompts, params


def _worker(rank, world, path, out_dir):
    import torch.distributed as dist

    from vllm_mps_b200.engine.distributed import ShardedEngine
    from vllm_mps_b200.engine.llm_engine import LLMEngine

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    eng = LLMEngine.from_model(_small_llama(), num_gpu_blocks=128, num_cpu_blocks=8,
                               max_batch_size=8, max_tokens_per_step=100000, mode="physical",
                               device=f"cuda:{rank}")
    sharded = ShardedEngine(eng)
    prompts, params = _workload()
    owner = sharded.add_requests(prompts, params)
    outs = sharded.run()
    torch.save({"owner": owner, "steps": sharded.steps,
                "tokens": {g: o.token_ids for g, o in outs.items()}},
               os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_engine_matches_single_engine():
    import torch.multiprocessing as mp

    from vllm_mps_b200.engine.llm_engine import LLMEngine

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs: the sharded engine's NCCL token gather runs one rank per GPU")
    world = 2
    d = tempfile.mkdtemp()
    mp.spawn(_worker, args=(world, os.path.join(d, "rdzv"), d), nprocs=world, join=True)
    res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]

    # Unsharded reference run on cuda:0, recording each decision's margin.
    eng = LLMEngine.from_model(_small_llama(), num_gpu_blocks=128, num_cpu_blocks=8,
                               max_batch_size=8, max_tokens_per_step=100000, mode="physical",
                               device="cuda:0")
    margins, last = {}, {}
    real_sample, real_update = eng.sampler.sample_rows, eng._update_sequences

    def spy_sample(logits, params, generator=None):
        last["l"] = logits.float()
        return real_sample(logits, params, generator)

    def spy_update(seq_ids, toks):
        top2 = torch.topk(last["l"], 2, dim=-1).values
        for r, sid in enumerate(seq_ids):
            margins.setdefault(sid, []).append(float(top2[r, 0] - top2[r, 1]))
        return real_update(seq_ids, toks)

    eng.sampler.sample_rows, eng._update_sequences = spy_sample, spy_update
    prompts, params = _workload()
    for p, sp in zip(prompts, params):
        eng.add_request(p, sp)
    while not eng.is_finished():
        eng.step()

    for r in range(world):
        assert res[r]["owner"] == res[0]["owner"] and res[r]["steps"] == res[0]["steps"]
    if world == 2:
        assert set(res[0]["owner"]) == {0, 1}
    for g in range(len(prompts)):
        ours = res[0]["tokens"][g]
        assert ours == res[-1]["tokens"][g]  # every rank assembled the same tokens
        ref = eng.get_output(g).token_ids
        assert len(ours) == len(ref) == params[g].max_tokens
        for t, (a, b) in enumerate(zip(ours, ref)):
            if a != b:
                assert margins[g][t] < 0.05, (g, t)
                break
