"""Sequence sharding and the per-step token gather, on CPU with gloo ranks.

The engine of each rank is replaced by a deterministic fake with the
engine's interface (add_request / step / is_finished), so these tests cover
the sharding, the gather records, the common stopping step and the failure
paths without a GPU.  Failures are made on the host: an engine that raises
(an allocator ``MemoryError`` injected at a given step) and a rank that never
joins the rendezvous.
"""

import datetime
import os
import time
import tempfile
from dataclasses import dataclass, field

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_mps_b200.core.sequence import SamplingParams
from vllm_mps_b200.engine.distributed import ShardedEngine, shard_requests


# ── sharding ─────────────────────────────────────────────────────────────────

def test_shard_requests_balances_and_is_deterministic():
    costs = [512, 40, 300, 300, 17, 4096, 80, 900, 64, 64, 1000]
    owner = shard_requests(costs, 3)
    assert owner == shard_requests(list(costs), 3)
    loads = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(3)]
    # The 4096-cost request dominates and gets a rank of its own; the others
    # split the rest within one request of each other.
    assert loads[owner[5]] == 4096
    rest = [l for i, l in enumerate(loads) if i != owner[5]]
    assert max(rest) - min(rest) <= max(c for c in costs if c != 4096)
    assert shard_requests([], 4) == []
    assert shard_requests([5, 5, 5, 5], 4) == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        shard_requests([1], 0)


def test_shard_requests_c4_shape_within_one_request_of_mean():
    import numpy as np

    rng = np.random.default_rng(0)
    prompts = np.clip(np.round(rng.lognormal(6, 1, 1024)), 16, 4096).astype(int)
    outs = rng.integers(16, 513, 1024)
    costs = (prompts + outs).tolist()
    owner = shard_requests(costs, 8)
    loads = np.bincount(owner, weights=costs, minlength=8)
    assert loads.max() - loads.mean() <= max(costs)
    assert loads.max() / loads.mean() < 1.01


# ── a fake engine with the engine's interface ────────────────────────────────

@dataclass
class _Out:
    request_id: int
    token_ids: list = field(default_factory=list)
    finished: bool = False


class FakeEngine:
    """Token t of a request = (sum(prompt) * 31 + 7 * t) % 1000; at most ``batch`` run per step."""

    def __init__(self, batch=4, fail_at_step=None, delay=None):
        self.batch, self.fail_at_step, self.delay = batch, fail_at_step, delay
        self.reqs, self.waiting, self.running = {}, [], []
        self.n_steps = 0

    def add_request(self, prompt, params):
        rid = len(self.reqs)
        self.reqs[rid] = (list(prompt), params.max_tokens, _Out(rid))
        self.waiting.append(rid)
        return rid

    def is_finished(self):
        return not self.waiting and not self.running

    def step(self):
        if self.fail_at_step is not None and self.n_steps == self.fail_at_step:
            raise MemoryError("BlockAllocator [gpu]: out of memory. 0 free blocks remaining.")
        if self.delay is not None:
            time.sleep(self.delay(self.n_steps))
        self.n_steps += 1
        while self.waiting and len(self.running) < self.batch:
            self.running.append(self.waiting.pop(0))
        outs = []
        for rid in list(self.running):
            prompt, max_tokens, out = self.reqs[rid]
            out.token_ids.append(expected_token(prompt, len(out.token_ids)))
            out.finished = len(out.token_ids) >= max_tokens
            if out.finished:
                self.running.remove(rid)
            outs.append(_Out(rid, list(out.token_ids), out.finished))
        return outs


def expected_token(prompt, t):
    return (sum(prompt) * 31 + 7 * t) % 1000


def _workload(n=13):
    prompts = [[i, i + 1, 3 * i] * (1 + i % 4) for i in range(n)]
    params = [SamplingParams(temperature=0.0, max_tokens=1 + (5 * i) % 9) for i in range(n)]
    return prompts, params


# ── gloo ranks ────────────────────────────────────────────────────────────────

def _init(rank, world, path, timeout_s=20):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("gloo", init_method=f"file://{path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _gather_worker(rank, world, path, result_dir, every=1):
    _init(rank, world, path)
    prompts, params = _workload()
    eng = ShardedEngine(FakeEngine(batch=3), gather_every=every)
    owner = eng.add_requests(prompts, params)
    outs = eng.run()
    res = {"owner": owner, "steps": eng.steps,
           "tokens": {g: o.token_ids for g, o in outs.items()},
           "finished": {g: o.finished for g, o in outs.items()}}
    torch.save(res, os.path.join(result_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def _spawn(fn, world, *args):
    d = tempfile.mkdtemp()
    path = os.path.join(d, "rdzv")
    mp.spawn(fn, args=(world, path, d, *args), nprocs=world, join=True)
    return d


@pytest.mark.parametrize("world,every", [(1, 1), (2, 1), (2, 3)])
def test_gather_assembles_every_request_on_every_rank(world, every):
    """Every rank assembles every request's tokens, in order, whether the ranks
    gather after every step or buffer ``every`` steps between gathers."""
    d = _spawn(_gather_worker, world, every)
    res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    prompts, params = _workload()
    for r in range(world):
        assert res[r]["owner"] == res[0]["owner"]
        assert res[r]["steps"] == res[0]["steps"]  # same collective count on every rank
        assert res[r]["steps"] % every == 0        # the run ends at a gather
        for g, p in enumerate(prompts):
            want = [expected_token(p, t) for t in range(params[g].max_tokens)]
            assert res[r]["tokens"][g] == want, (r, g)
            assert res[r]["finished"][g]
    if world == 2:
        assert set(res[0]["owner"]) == {0, 1}


def _oom_worker(rank, world, path, result_dir):
    _init(rank, world, path, timeout_s=5)
    prompts, params = _workload()
    eng = ShardedEngine(FakeEngine(batch=3, fail_at_step=2 if rank == 1 else None))
    eng.add_requests(prompts, params)
    outcome = "finished"
    try:
        eng.run()
    except MemoryError:
        outcome = "oom"
    except Exception as e:  # the peer's gather fails once rank 1 has left
        outcome = "peer-error:" + type(e).__name__
    with open(os.path.join(result_dir, f"r{rank}.txt"), "w") as f:
        f.write(outcome)
    if outcome == "oom":
        os._exit(0)  # leaves without entering the next collective
    dist.destroy_process_group()


def test_allocator_oom_on_one_rank_ends_the_other_rank_with_an_error():
    d = _spawn(_oom_worker, 2)
    r0 = open(os.path.join(d, "r0.txt")).read()
    r1 = open(os.path.join(d, "r1.txt")).read()
    assert r1 == "oom"
    assert r0.startswith("peer-error:"), r0


def _lonely_worker(rank, world, path, result_dir):
    try:
        _init(rank, world, path, timeout_s=2)
        outcome = "joined"
    except Exception as e:
        outcome = "timeout:" + type(e).__name__
    with open(os.path.join(result_dir, "lonely.txt"), "w") as f:
        f.write(outcome)


def test_rendezvous_times_out_when_a_rank_never_joins():
    d = tempfile.mkdtemp()
    path = os.path.join(d, "rdzv")
    # One process of a world of two: the second rank never arrives.
    mp.spawn(_lonely_entry, args=(path, d), nprocs=1, join=True)
    assert open(os.path.join(d, "lonely.txt")).read().startswith("timeout:")


def _lonely_entry(_i, path, d):
    _lonely_worker(0, 2, path, d)


def _capacity_worker(rank, world, path, result_dir):
    _init(rank, world, path)
    prompts, params = _workload(6)
    eng = ShardedEngine(FakeEngine(batch=4), capacity=2)
    eng.add_requests(prompts, params)
    try:
        eng.run()
        outcome = "ran"
    except RuntimeError as e:
        outcome = "capacity" if "capacity" in str(e) else "other"
    with open(os.path.join(result_dir, f"r{rank}.txt"), "w") as f:
        f.write(outcome)
    dist.destroy_process_group()


def test_record_capacity_is_enforced_before_the_collective():
    d = _spawn(_capacity_worker, 1)
    assert open(os.path.join(d, "r0.txt")).read() == "capacity"


def _max_steps_worker(rank, world, path, result_dir, every):
    _init(rank, world, path)
    prompts, params = _workload()
    eng = ShardedEngine(FakeEngine(batch=3), gather_every=every)
    eng.add_requests(prompts, params)
    outs = eng.run(max_steps=6)
    torch.save({"steps": eng.steps, "tokens": {g: o.token_ids for g, o in outs.items()}},
               os.path.join(result_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_max_steps_ends_on_a_gather_without_losing_buffered_tokens():
    """run(max_steps) forces a gather on its last step, so tokens buffered
    between gathers reach every rank: 6 steps with gathers every 4 steps give
    the same tokens as 6 steps with a gather after each."""
    got = {}
    for every in (1, 4):
        d = _spawn(_max_steps_worker, 2, every)
        got[every] = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(2)]
    for r in range(2):
        assert got[4][r]["steps"] == got[1][r]["steps"] == 6
        assert got[4][r]["tokens"] == got[1][0]["tokens"]
    assert any(got[1][0]["tokens"].values())


def _alternating_worker(rank, world, path, result_dir):
    _init(rank, world, path)
    prompts = [[rank + 1]] * 4
    params = [SamplingParams(temperature=0.0, max_tokens=12)] * 4
    # Rank r is slow on the steps of parity r: in lockstep every step would
    # cost the slow rank's 40 ms on both ranks.
    eng = ShardedEngine(FakeEngine(batch=4, delay=lambda s: 0.04 if s % 2 == rank else 0.0))
    eng.add_requests(prompts, params)
    t0 = time.perf_counter()
    eng.run()
    torch.save({"wall": time.perf_counter() - t0, "gather_s": eng.gather_seconds,
                "steps": eng.steps, "tokens": {g: o.token_ids for g, o in eng.outputs.items()}},
               os.path.join(result_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_gathers_overlap_the_local_steps():
    """Gathers are read back one gather late, so a rank that is ahead keeps
    stepping: with the slow steps alternating between the ranks, each rank
    waits in gathers for much less than the 6 x 40 ms a lockstep exchange
    would cost it."""
    d = _spawn(_alternating_worker, 2)
    res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(2)]
    assert res[0]["steps"] == res[1]["steps"]
    assert res[0]["tokens"] == res[1]["tokens"]
    assert all(len(t) == 12 for t in res[0]["tokens"].values())
    for r in range(2):
        assert res[r]["gather_s"] < 0.12, res[r]
