"""Bit-exact slotting against the reference's recorded operation streams.

``tests/golden/slots_trace.npz`` holds a 600-op stream (allocate, append,
free, fork, swap_out, swap_in, and appends that hit out-of-memory) run
through the reference ``KVCacheManager``, with every live block table and
the free counts after each op.  ``sched_trace*.npz`` hold request streams
through the reference ``Scheduler`` (per step: scheduled sequence ids,
preempted groups, token counts, every block table, queue lengths), one of
them ending in the reference's step-4 ``MemoryError``.  Replaying them here
must give identical tables, ids and counts.
"""

import ast

import numpy as np
import pytest

from conftest import load_golden
from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
from vllm_mps_b200.core.sequence import SamplingParams, Sequence, SequenceGroup, SequenceStatus
from vllm_mps_b200.engine.scheduler import Scheduler


def test_kv_cache_manager_replays_reference_op_stream():
    d = load_golden("slots_trace.npz")
    m = KVCacheManager(int(d["gpu"]), int(d["cpu"]))
    for op, (a, b), tables, (fg, fc) in zip(d["ops"], d["args"], d["tables"], d["free"]):
        op = str(op)
        if op == "allocate":
            m.allocate(int(a))
        elif op in ("append", "append_oom"):
            for _ in range(int(b)):
                m.append_slot(int(a))
            if op == "append_oom":
                with pytest.raises(MemoryError):
                    m.append_slot(int(a))
        elif op == "free":
            m.free(int(a))
        elif op == "fork":
            m.fork(int(a), int(b))
        elif op == "swap_out":
            m.swap_out(int(a))
        elif op == "swap_in":
            m.swap_in(int(a))
        else:
            raise AssertionError(op)
        snap = {s: m.get_block_table(s) for s in sorted(m.get_all_seq_ids())}
        assert snap == ast.literal_eval(str(tables)), op
        assert (m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()) == (int(fg), int(fc))


@pytest.mark.parametrize("name", ["sched_trace.npz", "sched_trace_oom.npz"])
def test_scheduler_replays_reference_request_stream(name):
    d = load_golden(name)
    rng = np.random.default_rng(int(d["arrival_seed"]))
    # The generator drew the request table first, then arrivals per step.
    reqs = []
    for i in range(24):
        plen = int(rng.integers(1, 60))
        mx = int(rng.integers(1, 40))
        reqs.append((i, plen, mx))
    assert reqs == [tuple(map(int, r)) for r in d["reqs"]]
    kv = KVCacheManager(int(d["gpu"]), int(d["cpu"]))
    sched = Scheduler(kv, max_batch_size=int(d["max_batch"]), max_tokens_per_step=int(d["max_tokens"]))
    pending = list(reqs)
    steps = [str(x) for x in d["steps"]]
    for step, expect in enumerate(steps):
        for _ in range(int(rng.integers(0, 3))):
            if pending:
                gid, plen, mx = pending.pop(0)
                p = SamplingParams(temperature=0.0, max_tokens=mx)
                sched.add_request(SequenceGroup(gid, [Sequence(gid, "", list(range(plen)), p)], p))
        if expect.startswith("('MemoryError"):
            with pytest.raises(MemoryError):
                sched.schedule()
            return
        out = sched.schedule()
        scheduled = [s.seq_id for g in out.scheduled_groups for s in g.get_seqs(SequenceStatus.RUNNING)]
        preempted = [g.group_id for g in out.preempted_groups]
        tables = {s: kv.get_block_table(s) for s in sorted(kv.get_all_seq_ids())}
        for g in out.scheduled_groups:
            for s in g.get_seqs(SequenceStatus.RUNNING):
                s.add_token(step % 1000)
                if s.is_finished():
                    sched.mark_finished(s.seq_id)
        got = (scheduled, preempted, out.num_batched_tokens, out.num_scheduled_seqs, tables,
               sched.get_num_waiting(), sched.get_num_running(), sched.get_num_preempted())
        assert got == ast.literal_eval(expect), f"step {step}"
