"""Host-side bookkeeping: the behaviours the reference's unit tests pin.

Covers the contracts tested by the reference's tests/test_block.py,
test_block_allocator.py, test_block_table.py, test_kv_cache_manager.py,
test_sequence.py and test_scheduler.py (block invariants, FIFO allocation,
lazy page tables, fork/swap accounting, request state, admission/preemption)
on this package's classes.  Bit-exact agreement with the reference's own
classes is in test_slot_traces.py.
"""

import pytest

from vllm_mps_b200.config import BLOCK_SIZE
from vllm_mps_b200.core.block import PhysicalBlock
from vllm_mps_b200.core.block_allocator import BlockAllocator, BlockAllocatorType
from vllm_mps_b200.core.block_table import BlockTable
from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
from vllm_mps_b200.core.sequence import SamplingParams, Sequence, SequenceGroup, SequenceStatus
from vllm_mps_b200.engine.scheduler import Scheduler


# ── PhysicalBlock ────────────────────────────────────────────────────────────

def test_block_defaults_and_flags():
    b = PhysicalBlock(3)
    assert (b.ref_count, b.num_tokens, b.block_size) == (0, 0, BLOCK_SIZE)
    assert b.is_free and not b.is_full and b.num_empty_slots == BLOCK_SIZE
    b.add_tokens(BLOCK_SIZE)
    assert b.is_full and b.num_empty_slots == 0


def test_block_errors_and_reset():
    b = PhysicalBlock(0)
    with pytest.raises(ValueError):
        b.decrement_ref()
    with pytest.raises(ValueError):
        b.add_tokens(BLOCK_SIZE + 1)
    b.increment_ref()
    b.add_tokens(5)
    b.reset()
    assert (b.ref_count, b.num_tokens) == (0, 0)
    assert "block 0" in repr(b)


# ── BlockAllocator ───────────────────────────────────────────────────────────

def test_allocator_fifo_order_and_reuse_after_fresh_ids():
    a = BlockAllocator(BlockAllocatorType.GPU, 4)
    got = [a.allocate().block_id for _ in range(3)]
    assert got == [0, 1, 2]
    a.free(a.block(1))
    # The freed id goes to the back: fresh id 3 comes first.
    assert a.allocate().block_id == 3
    assert a.allocate().block_id == 1
    with pytest.raises(MemoryError):
        a.allocate()


def test_allocator_counts_and_fork():
    a = BlockAllocator(BlockAllocatorType.CPU, 5)
    b = a.allocate()
    assert a.get_num_free_blocks() == 4 and a.get_num_used_blocks() == 1
    assert a.get_utilisation() == pytest.approx(0.2)
    a.fork(b)
    assert b.ref_count == 2
    a.free(b)
    assert a.get_num_free_blocks() == 4  # still referenced
    a.free(b)
    assert a.get_num_free_blocks() == 5 and b.num_tokens == 0
    with pytest.raises(ValueError):
        a.fork(PhysicalBlock(99))
    assert a.get_all_free_block_ids()[-1] == b.block_id


# ── BlockTable ───────────────────────────────────────────────────────────────

def test_block_table_lazy_allocation_and_spill():
    a = BlockAllocator(BlockAllocatorType.GPU, 10)
    t = BlockTable(0, a)
    assert t.is_empty() and t.num_blocks() == 0
    for _ in range(BLOCK_SIZE):
        t.append_slot()
    assert t.num_blocks() == 1 and t.get_last_block().is_full
    t.append_slot()
    assert t.num_blocks() == 2 and t.num_tokens() == BLOCK_SIZE + 1
    ids = t.get_all_physical_block_ids()
    assert len(set(ids)) == 2
    with pytest.raises(IndexError):
        t.get_block(5)
    t.free_all()
    assert t.is_empty() and a.get_num_free_blocks() == 10
    with pytest.raises(IndexError):
        t.get_last_block()


def test_block_tables_are_disjoint_and_oom_propagates():
    a = BlockAllocator(BlockAllocatorType.GPU, 2)
    t1, t2 = BlockTable(1, a), BlockTable(2, a)
    t1.append_slot()
    t2.append_slot()
    assert set(t1.get_all_physical_block_ids()).isdisjoint(t2.get_all_physical_block_ids())
    for _ in range(BLOCK_SIZE - 1):
        t1.append_slot()
    with pytest.raises(MemoryError):
        t1.append_slot()


# ── KVCacheManager ───────────────────────────────────────────────────────────

def test_kv_manager_lifecycle():
    m = KVCacheManager(16, 8)
    assert m.get_num_free_gpu_blocks() == 16 and m.get_all_seq_ids() == []
    m.allocate(0)
    with pytest.raises(ValueError):
        m.allocate(0)
    for _ in range(BLOCK_SIZE + 1):
        m.append_slot(0)
    assert m.get_num_free_gpu_blocks() == 14 and len(m.get_block_table(0)) == 2
    assert m.can_allocate(0, BLOCK_SIZE - 1) and not m.can_allocate(1, 17 * BLOCK_SIZE)
    m.free(0)
    assert m.get_num_free_gpu_blocks() == 16
    for call in (m.free, m.append_slot, m.get_block_table, m.swap_out, m.swap_in):
        with pytest.raises(KeyError):
            call(99)


def test_kv_manager_fork_and_swap_accounting():
    m = KVCacheManager(16, 8)
    m.allocate(0)
    for _ in range(BLOCK_SIZE):
        m.append_slot(0)
    m.fork(0, 1)
    assert m.get_block_table(0) == m.get_block_table(1)
    assert all(m.gpu_allocator.block(b).ref_count == 2 for b in m.get_block_table(0))
    with pytest.raises(ValueError):
        m.fork(0, 1)
    m.free(0)
    assert 1 in m.get_all_seq_ids() and m.get_num_free_gpu_blocks() == 15
    m.allocate(2)
    for _ in range(20):
        m.append_slot(2)
    gpu, cpu = m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()
    m.swap_out(2)
    assert (m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()) == (gpu + 2, cpu - 2)
    m.swap_in(2)
    assert (m.get_num_free_gpu_blocks(), m.get_num_free_cpu_blocks()) == (gpu, cpu)
    for _ in range(4):  # still fits the half-filled second block
        m.append_slot(2)
    assert m.get_num_free_gpu_blocks() == gpu
    m.free(2)
    m.free(1)
    assert m.get_gpu_utilisation() == 0.0 and m.get_cpu_utilisation() == 0.0


def test_swap_space_hook_receives_block_pairs():
    calls = []

    class Recorder:
        def copy_out(self, g, c):
            calls.append(("out", list(g), list(c)))

        def copy_in(self, c, g):
            calls.append(("in", list(c), list(g)))

    m = KVCacheManager(8, 8, swap_space=Recorder())
    m.allocate(0)
    for _ in range(BLOCK_SIZE + 1):
        m.append_slot(0)
    m.swap_out(0)
    m.swap_in(0)
    assert calls == [("out", [0, 1], [0, 1]), ("in", [0, 1], [2, 3])]


# ── Sequence / SamplingParams ────────────────────────────────────────────────

def test_sampling_params_validation():
    for kw in ({"temperature": -1}, {"top_k": -1}, {"top_p": 0.0}, {"top_p": 1.5}, {"max_tokens": 0}):
        with pytest.raises(ValueError):
            SamplingParams(**kw)
    assert SamplingParams().max_tokens == 128


def test_sequence_state_machine():
    s = Sequence(7, "p", [1, 2, 3], SamplingParams(max_tokens=2))
    assert s.status == SequenceStatus.WAITING and s.get_prompt_len() == 3
    s.add_token(9)
    assert s.get_total_len() == 4 and s.get_output_len() == 1 and not s.is_finished()
    s.add_token(10)
    assert s.is_finished() and s.get_last_token_id() == 10
    with pytest.raises(IndexError):
        Sequence(1, "", [], SamplingParams()).get_last_token_id()
    g = SequenceGroup(1, [s, Sequence(8, "q", [1], SamplingParams())], SamplingParams())
    assert g.get_num_seqs() == 2 and g.get_num_seqs(SequenceStatus.FINISHED) == 1
    assert not g.is_finished() and g.get_max_total_len() == 5


# ── Scheduler ────────────────────────────────────────────────────────────────

def _group(gid, plen=4, max_tokens=10):
    p = SamplingParams(max_tokens=max_tokens)
    return SequenceGroup(gid, [Sequence(gid * 100, "p", list(range(plen)), p)], p)


def test_scheduler_admission_limits_and_fifo():
    sched = Scheduler(KVCacheManager(32, 16), max_batch_size=2, max_tokens_per_step=512)
    out = sched.schedule()
    assert out.num_scheduled_seqs == 0
    groups = [_group(i, plen=2) for i in range(5)]
    for g in groups:
        sched.add_request(g)
    out = sched.schedule()
    assert out.scheduled_groups == groups[:2] and sched.get_num_waiting() == 3
    assert out.num_batched_tokens == 4


def test_scheduler_finish_frees_memory_and_token_budget():
    kv = KVCacheManager(32, 16)
    sched = Scheduler(kv, max_batch_size=8, max_tokens_per_step=10)
    sched.add_request(_group(0, plen=8))
    sched.add_request(_group(1, plen=8))
    out = sched.schedule()
    assert out.num_scheduled_seqs == 1  # second would exceed 10 tokens
    free = kv.get_num_free_gpu_blocks()
    sched.mark_finished(0)
    assert kv.get_num_free_gpu_blocks() > free and sched.get_num_running() == 0


def test_scheduler_preempts_when_no_block_is_left():
    kv = KVCacheManager(4, 4)
    sched = Scheduler(kv, max_batch_size=10, max_tokens_per_step=9999)
    g0 = _group(0, plen=BLOCK_SIZE * 4)  # fills every block exactly
    sched.add_request(g0)
    sched.schedule()
    out = sched.schedule()  # needs a 5th block for the next token
    assert out.preempted_groups == [g0] and sched.get_num_preempted() == 1
    assert kv.get_num_free_gpu_blocks() == 4 and kv.get_num_free_cpu_blocks() == 0


def test_scheduler_watermark_keeps_reserve():
    kv = KVCacheManager(10, 10)
    sched = Scheduler(kv, max_batch_size=8, max_tokens_per_step=9999, preempt_watermark=0.5)
    sched.add_request(_group(0, plen=BLOCK_SIZE * 4))
    sched.add_request(_group(1, plen=BLOCK_SIZE * 2))
    out = sched.schedule()
    # 4 blocks fit under the 5-block reserve line, the next 2 would not.
    assert [g.group_id for g in out.scheduled_groups] == [0]


def test_block_id_arrays_follow_appends_swaps_and_forks():
    """The int32 id arrays a decode step copies equal the block lists after
    every kind of change: appends across page boundaries, swap out and in
    (new physical blocks), fork (shared blocks) and free."""
    import numpy as np

    from vllm_mps_b200.core.kv_cache_manager import KVCacheManager

    m = KVCacheManager(64, 32)

    def same(sid):
        want = m.get_block_table(sid)
        got = m.get_block_ids(sid)
        assert got.dtype == np.int32 and got.tolist() == want
        assert not got.flags.writeable

    m.allocate(0)
    m.allocate(1)
    for t in range(300):  # 19 pages, past the array's first capacity of 16
        m.append_slot(0)
        if t % 3 == 0:
            m.append_slot(1)
        same(0)
        same(1)
    m.swap_out(0)
    same(0)
    m.swap_in(0)
    same(0)
    m.append_slot(0)
    same(0)
    m.fork(1, 2)
    same(2)
    for _ in range(40):
        m.append_slot(2)
    same(2)
    same(1)
    m.free(0)
    m.allocate(0)
    same(0)
    m.append_slot(0)
    same(0)


def test_bulk_slot_appends_equal_single_appends():
    """append_slots(n) takes the same blocks, in the same FIFO order, with the
    same fills as n calls of append_slot -- including when the pool runs out
    part-way (the MemoryError comes at the same slot, with the same state)."""
    import numpy as np

    rng = np.random.default_rng(3)
    a, b = KVCacheManager(40, 8), KVCacheManager(40, 8)
    live = []
    for step in range(200):
        op = rng.integers(0, 4)
        if op == 0 or not live:
            sid = step
            a.allocate(sid)
            b.allocate(sid)
            live.append(sid)
        elif op == 1:
            sid = live[rng.integers(len(live))]
            n = int(rng.integers(1, 60))
            ea = eb = None
            try:
                a.append_slots(sid, n)
            except MemoryError as e:
                ea = e
            try:
                for _ in range(n):
                    b.append_slot(sid)
            except MemoryError as e:
                eb = e
            assert (ea is None) == (eb is None)
        elif op == 2:
            sid = live.pop(rng.integers(len(live)))
            a.free(sid)
            b.free(sid)
        else:
            sid = live[rng.integers(len(live))]
            assert a.free_slots_in_last_block(sid) == b.free_slots_in_last_block(sid)
        for sid in live:
            assert a.get_block_table(sid) == b.get_block_table(sid)
            assert a.num_tokens(sid) == b.num_tokens(sid)
        assert a.gpu_allocator.get_all_free_block_ids() == b.gpu_allocator.get_all_free_block_ids()
        assert np.array_equal(a.gpu_allocator.counters.fill, b.gpu_allocator.counters.fill)
        assert np.array_equal(a.gpu_allocator.counters.ref, b.gpu_allocator.counters.ref)
