#!/usr/bin/env python
"""Throughput of the paged decode-attention step on B200 (one JSON line on stdout).

Workload (config 1 of the north star, the single-GPU microbench): one decode
step of one attention layer for a batch of 64 sequences -- 32 query heads,
4 kv heads, head_dim 64, fp16, context lengths uniform in [1, 2048], block
tables a random permutation of a 16384-block pool.  A "step" is the hot path
of ``PagedAttentionLayer._forward_batch`` between its projections: RoPE on
Q/K, the K/V write into the pool slot, and paged GQA decode attention
(``vmps_paged_decode_step``: one kernel launch per step).

Sequences are independent, so ``--gpus N`` shards them: every rank runs its
own 64-sequence batch on its own pool (weak scaling, no collective on the
data path; one all-reduce after the timed region takes the max time).

Measurement:
* ``value``: tokens/s of the whole job, inputs resident in HBM, CUDA-graph
  replays of the step timed with CUDA events (max over ranks).  Eight pool
  replicas (8 x 256 MiB, 8 x ~67 MB touched) are rotated so successive steps
  never hit in the 126 MB L2.
* ``e2e``: the same metric through the public Python API
  (``vllm_mps_b200.kernels.paged_decode_step``) with the per-step inputs in
  pinned host memory, copied to the device, and the output copied back,
  inside the timed region.  The KV pool is device-resident state.
* ``roofline``: the attention kernel timed alone with CUDA events (graphs of
  8 launches); algorithmic bytes = K/V rows read + q + out + block-table
  entries + seq_lens; peak = measured HBM copy bandwidth (MEASURED_PEAKS.json).
* ``cpu_baseline``: the C oracle (oracle/vmps_oracle.c, a port of the
  reference's CPU path) on the host cores, rank 0, N=1 only.

``--impl reference`` times that CPU implementation alone (the reference is
Python + Metal; its CPU path is what runs off Apple hardware).
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (B, n_q, n_kv, D, dtype, ctx_lo, ctx_hi, num_blocks, replicas, description)
    "c1": (64, 32, 4, 64, "float16", 1, 2048, 16384, 8,
           "C1 single-layer paged decode step: batch 64, 32 q / 4 kv heads, head_dim 64, "
           "fp16, ctx U[1,2048], block_size 16, permuted 16384-block pool"),
    "c2layer": (256, 32, 8, 128, "bfloat16", 128, 4224, 36000, 2,
                "C2 single layer: Llama-3-8B attention (32 q / 8 kv heads, head_dim 128), bf16, "
                "batch 256, ctx U[128,4224] (prompts U[128,4096] + 128 steps), block_size 16, "
                "permuted 36000-block pool"),
    "c3": (4, 64, 8, 128, "float16", 131072, 131072, 32768 + 64, 2,
           "C3 long-context split-K decode: batch 4 x 131072, 64 q / 8 kv heads, "
           "head_dim 128, fp16, permuted 32832-block pool"),
}
BLOCK = 16


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


KERNEL_SOURCES = ("vllm_mps_b200/csrc/paged_decode.cu", "vllm_mps_b200/csrc/vmps_common.cuh")


def kernel_source_hash():
    """sha256 over the decode kernel's source files (what an ncu capture measured)."""
    import hashlib

    h = hashlib.sha256()
    for rel in KERNEL_SOURCES:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def profile_traffic(cfg_name):
    """ncu DRAM bytes per launch of the decode kernel on ``cfg_name``, or None.

    profiles/decode_traffic.json holds, per config, the read + write bytes of
    one launch from an ncu capture together with the sha256 of the kernel
    sources it was captured from; after any change to those sources the
    stored figure no longer describes the kernel and None is returned.
    """
    try:
        with open(os.path.join(ROOT, "profiles", "decode_traffic.json")) as f:
            rec = json.load(f).get(cfg_name)
    except (OSError, ValueError):
        return None
    if not rec or rec.get("kernel_source_sha256") != kernel_source_hash():
        return None
    return int(rec["traffic_bytes_per_launch"])


def make_host_workload(cfg, seed):
    B, n_q, n_kv, D, dt, lo, hi, nb, R, _ = cfg
    rng = np.random.default_rng(seed)
    ctx = rng.integers(lo, hi + 1, size=B).astype(np.int64)
    pages = (ctx + BLOCK - 1) // BLOCK
    maxb = int(pages.max())
    tables = []
    for _ in range(R):
        perm = rng.permutation(nb)
        bt = np.zeros((B, maxb), np.int32)
        off = 0
        for i, p in enumerate(pages):
            bt[i, :p] = perm[off:off + p]
            off += p
        tables.append(bt)
    return ctx, pages, tables


def decode_config(cfg, ctx, world):
    """The ``config`` object of a decode-step line (identical on both arms)."""
    B, lo, hi, desc = cfg[0], cfg[5], cfg[6], cfg[9]
    return {"workload": desc, "global_batch": B * world, "seq_len": "U[%d,%d]" % (lo, hi),
            "sum_ctx_per_rank": int(ctx.sum()), "parallelism": f"sequence-sharded x{world}"}


def alg_bytes(cfg, ctx, pages, fused=False):
    """Bytes one launch must move: the K/V history, q in and out, tables, lengths.

    ``fused`` (the decode step): plus the new token's k and v read, its
    rotated K and V written to the slot, and positions and slots read.
    """
    B, n_q, n_kv, D = cfg[0], cfg[1], cfg[2], cfg[3]
    kv = int(ctx.sum()) * n_kv * D * 2 * 2
    base = kv + 2 * B * n_q * D * 2 + int(pages.sum()) * 4 + 4 * B
    if fused:
        base += 2 * (2 * B * n_kv * D * 2) + 2 * 4 * B
    return base


class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while running."""

    NAMES = {
        "nvmlClocksEventReasonGpuIdle": "gpu_idle",
        "nvmlClocksEventReasonApplicationsClocksSetting": "applications_clocks_setting",
        "nvmlClocksEventReasonSwPowerCap": "sw_power_cap",
        "nvmlClocksEventReasonHwSlowdown": "hw_slowdown",
        "nvmlClocksEventReasonSyncBoost": "sync_boost",
        "nvmlClocksEventReasonSwThermalSlowdown": "sw_thermal_slowdown",
        "nvmlClocksEventReasonHwThermalSlowdown": "hw_thermal_slowdown",
        "nvmlClocksEventReasonHwPowerBrakeSlowdown": "hw_power_brake_slowdown",
    }

    def __init__(self, index, period=0.01):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period = period
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report nulls
            log(f"clock sampling unavailable: {e}")
            self.max_mhz = None

    def _sample(self):
        nv = self.nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        for attr, name in self.NAMES.items():
            if mask & getattr(nv, attr, 0):
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": []}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def cpu_baseline(cfg, ctx, tables, budget_s=10.0):
    """C oracle (port of the reference's CPU path) on all host cores, bounded sample."""
    from oracle import c_oracle
    from oracle.paged_attention_oracle import f32_to_bits, rope_inv_freq

    c_oracle.build()
    B, n_q, n_kv, D, dt, lo, hi, nb, R, _ = cfg
    rng = np.random.default_rng(99)
    pool = f32_to_bits(rng.standard_normal((nb, 2, BLOCK, n_kv, D), dtype=np.float32), dt)
    q = f32_to_bits(rng.standard_normal((B, n_q, D), dtype=np.float32), dt)
    k = f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), dt)
    v = f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), dt)
    inv = rope_inv_freq(D, 10000.0)
    threads = os.cpu_count() or 1
    # Warm-up, then as many full steps as fit in the budget (at least one).
    c_oracle.decode_step(q, k, v, ctx - 1, ctx, tables[0], pool, inv, dt, threads=threads)
    t0 = time.perf_counter()
    n = 0
    while True:
        c_oracle.decode_step(q, k, v, ctx - 1, ctx, tables[n % len(tables)], pool, inv, dt,
                             threads=threads)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt_s = time.perf_counter() - t0
    return {"value": B * n / dt_s, "unit": "tokens/s", "cores": c_oracle.max_threads(),
            "kind": "port",
            "sample": f"{n} full steps of the same workload ({B} seqs, sum ctx {int(ctx.sum())}) "
                      f"in {dt_s:.1f} s, C oracle (oracle/vmps_oracle.c), OpenMP"}


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return 0
    from oracle import c_oracle
    from oracle.paged_attention_oracle import f32_to_bits, rope_inv_freq

    c_oracle.build()
    B, n_q, n_kv, D, dt, lo, hi, nb, R, desc = cfg
    ctx, pages, tables = make_host_workload(cfg, seed=1000)
    rng = np.random.default_rng(99)
    pool = f32_to_bits(rng.standard_normal((nb, 2, BLOCK, n_kv, D), dtype=np.float32), dt)
    q = f32_to_bits(rng.standard_normal((B, n_q, D), dtype=np.float32), dt)
    k = f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), dt)
    v = f32_to_bits(rng.standard_normal((B, n_kv, D), dtype=np.float32), dt)
    inv = rope_inv_freq(D, 10000.0)
    threads = os.cpu_count() or 1

    def step(i, sel):
        c_oracle.decode_step(q[sel], k[sel], v[sel], ctx[sel] - 1, ctx[sel], tables[i % R][sel],
                             pool, inv, dt, threads=threads)

    # Size the per-step sample so the whole run stays within ~3 minutes.
    full = np.arange(B)
    t0 = time.perf_counter()
    step(0, full)
    t_full = time.perf_counter() - t0
    total = args.steps + args.warmup
    budget = 150.0
    sel = full
    if t_full * total > budget:
        keep = max(1, int(B * budget / (t_full * total)))
        sel = np.sort(np.random.default_rng(5).choice(B, size=keep, replace=False))
    for i in range(args.warmup):
        step(i, sel)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i, sel)
    el = time.perf_counter() - t0
    toks = len(sel) * args.steps
    val = toks / el
    line = {
        "metric": "decode tokens/s", "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if dt == "bfloat16" else "f16",
        "data": "synthetic (seeded)", "impl": "reference",
        "config": decode_config(cfg, ctx, world),
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": c_oracle.max_threads(),
                         "kind": "port",
                         "sample": f"{len(sel)} of {B} sequences per step (sum ctx "
                                   f"{int(ctx[sel].sum())}), C oracle oracle/vmps_oracle.c"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def decode_leg(args, cfg_name, rank, world, local_rank, cpu_base=True):
    """One decode-step config (c1/c2layer/c3): the record on rank 0, None elsewhere."""
    cfg = CONFIGS[cfg_name]
    import torch

    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, n_q, n_kv, D, dt, lo, hi, nb, R, desc = cfg
    tdt = getattr(torch, dt)
    ctx, pages, tables = make_host_workload(cfg, seed=1000 + rank)
    maxb = tables[0].shape[1]
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    pools = [torch.randn((nb, 2, BLOCK, n_kv, D), generator=g, device=dev, dtype=torch.float32)
             .to(tdt) for _ in range(R)]
    qs = [torch.randn((B, n_q, D), generator=g, device=dev, dtype=torch.float32).to(tdt)
          for _ in range(R)]
    k = torch.randn((B, n_kv, D), generator=g, device=dev, dtype=torch.float32).to(tdt)
    v = torch.randn((B, n_kv, D), generator=g, device=dev, dtype=torch.float32).to(tdt)
    pos_np = (ctx - 1).astype(np.int32)
    pos = torch.from_numpy(pos_np).to(dev)
    sl = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    bts = [torch.from_numpy(t).to(dev) for t in tables]
    slots_np = [np.array([t[i, p // BLOCK] * BLOCK + p % BLOCK for i, p in enumerate(pos_np)],
                         np.int32) for t in tables]
    slots = [torch.from_numpy(s).to(dev) for s in slots_np]
    inv = rope_inv_freq(D, 10000.0).to(dev)
    outs = [torch.empty((B, n_q, D), dtype=tdt, device=dev) for _ in range(R)]
    ws = K.DecodeWorkspace()

    def step(r):
        K.paged_decode_step(qs[r], k, v, pos, slots[r], inv, pools[r], bts[r], sl,
                            out=outs[r], workspace=ws)

    def attn(r):
        K.paged_decode_attention(qs[r], pools[r], bts[r], sl, out=outs[r], workspace=ws)

    # Eager warm-up (loads the library, sizes the workspace), then capture the
    # steps as CUDA graphs: one graph of R consecutive steps (one per replica,
    # chained with programmatic dependent launch, as a serving loop would
    # replay them) and single-step graphs for a remainder of K % R steps.
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for r in range(R):
            step(r)
            attn(r)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)

    def capture(fn_list):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for fn in fn_list:
                fn()
        return gr

    # The timed K steps are ONE graph of K PDL-chained launches (replicas
    # rotating), so the timed region is one replay with no graph boundary
    # between steps -- the steady state a serving loop sees.  The warm-up
    # steps are a graph of their own.
    # The timed graph starts and ends with event-record nodes (external
    # events), so the events stamp the first launch's start and the last
    # launch's end on the device; events recorded on the stream around the
    # replay also see the graph's submission latency, reported beside it.
    graphs = {}
    ev_in = (torch.cuda.Event(enable_timing=True, external=True),
             torch.cuda.Event(enable_timing=True, external=True))

    def run_steps(n, timed=False):
        if (n, timed) not in graphs:
            fns = [lambda i=i: step(i % R) for i in range(n)]
            if timed:
                fns = [ev_in[0].record] + fns + [ev_in[1].record]
            graphs[(n, timed)] = capture(fns)
            torch.cuda.synchronize(dev)
        graphs[(n, timed)].replay()

    run_steps(args.warmup)
    run_steps(args.steps, timed=True)
    g_attns = capture([lambda r=r: attn(r) for r in range(R)])
    torch.cuda.synchronize(dev)
    if K.error_word(dev):
        raise RuntimeError("device error word set during warm-up")

    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ── timed region: K steps ────────────────────────────────────────────────
    run_steps(args.warmup)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        e0.record()
        run_steps(args.steps, timed=True)
        e1.record()
        torch.cuda.synchronize(dev)
    barrier()
    t_step = max_over_ranks(ev_in[0].elapsed_time(ev_in[1]) * 1e-3)
    t_replay = max_over_ranks(e0.elapsed_time(e1) * 1e-3)

    # ── the attention kernel alone (roofline): R launches per graph replay,
    # CUDA events around every replay; duration per launch = replay time / R.
    n_k = max(args.steps // R, 20)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_k)]
    for _ in range(max(args.warmup // R, 3)):
        g_attns.replay()
    torch.cuda.synchronize(dev)
    for i in range(n_k):
        evs[i][0].record()
        g_attns.replay()
        evs[i][1].record()
    torch.cuda.synchronize(dev)
    t_kernel = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evs) * 1e-3 / R)

    # ── end to end through the public API with host buffers ───────────────────
    # Every step's inputs (q, k, v, positions, seq_lens, slot_mapping, block
    # table) are packed in one pinned host buffer and copied with one H2D
    # copy; the output comes back with one D2H copy.  Steps are pipelined the
    # way a serving loop runs them: the H2D of step i+1 and the D2H of step
    # i-1 run on two copy streams while step i computes (double-buffered
    # device staging and output).
    def pack(r):
        parts = [qs[r].cpu().contiguous().view(torch.uint8).reshape(-1),
                 k.cpu().contiguous().view(torch.uint8).reshape(-1),
                 v.cpu().contiguous().view(torch.uint8).reshape(-1),
                 torch.from_numpy(pos_np).view(torch.uint8),
                 torch.from_numpy(ctx.astype(np.int32)).view(torch.uint8),
                 torch.from_numpy(slots_np[r]).view(torch.uint8),
                 torch.from_numpy(np.ascontiguousarray(tables[r])).view(torch.uint8).reshape(-1)]
        offs, o = [], 0
        for t in parts:
            offs.append(o)
            o += (t.numel() + 255) // 256 * 256
        buf = torch.zeros(o, dtype=torch.uint8).pin_memory()
        for t, off in zip(parts, offs):
            buf[off:off + t.numel()].copy_(t)
        return buf, offs, [t.numel() for t in parts]

    packed = [pack(r) for r in range(R)]
    nbytes = packed[0][0].numel()
    offs, sizes = packed[0][1], packed[0][2]
    # Per step: the packed pinned inputs go to a device staging buffer with
    # kernels.stage_copy -- a kernel that is a link of the decode steps'
    # programmatic-dependent-launch chain, so it overlaps the step before it
    # and no copy-engine node ever feeds a decode step (which would cost that
    # step its early launch) -- then the decode step, then a copy-engine D2H
    # of the step's output on a copy stream.  Every step writes its own
    # device output buffer, so the chain never waits for a D2H.
    # Inputs are staged two steps per copy kernel: steps 2p+1 and 2p+2 in one
    # stage_copy right BEFORE step 2p's decode kernel (one extra link in the
    # chain per two steps).  The fused step reads its lengths and block tables
    # before its PDL wait, so the kernel just ahead of it must not be the one
    # writing them; here every step is at least one decode kernel behind its
    # copy.  Three pair slots keep a copy clear of the steps around it; the
    # host side holds each replica's packed inputs followed by the next's, so
    # a pair is one contiguous source.
    e2e_steps = min(args.steps, 512)
    stage0 = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    pair_slots = [torch.empty(2 * nbytes, dtype=torch.uint8, device=dev) for _ in range(3)]
    host_cat = torch.empty((R + 1) * nbytes, dtype=torch.uint8).pin_memory()
    for r in range(R + 1):
        host_cat[r * nbytes:(r + 1) * nbytes].copy_(packed[r % R][0])
    douts = [torch.empty((B, n_q, D), dtype=tdt, device=dev) for _ in range(e2e_steps)]
    houts = [torch.empty((B, n_q, D), dtype=tdt).pin_memory() for _ in range(2)]
    maxb_r = tables[0].shape[1]

    def views(buf):
        def sl(i):
            return buf[offs[i]:offs[i] + sizes[i]]
        return (sl(0).view(tdt).view(B, n_q, D), sl(1).view(tdt).view(B, n_kv, D),
                sl(2).view(tdt).view(B, n_kv, D), sl(3).view(torch.int32),
                sl(4).view(torch.int32), sl(5).view(torch.int32),
                sl(6).view(torch.int32).view(B, maxb_r))

    staged0 = views(stage0)
    staged_pairs = [(views(b[:nbytes]), views(b[nbytes:])) for b in pair_slots]

    def staged_for(i):
        if i == 0:
            return staged0
        p = (i - 1) // 2
        return staged_pairs[p % 3][(i - 1) % 2]

    s_d2h = torch.cuda.Stream(dev)
    k_done = [torch.cuda.Event() for _ in range(2)]

    def run_pipeline(n, first=None, last=None):
        comp = torch.cuda.current_stream(dev)
        if first is not None:
            first.record(comp)
        # The first step's inputs go by copy engine (a full dependency): a
        # stage copy lets the next launch start at once, so a stage copy just
        # ahead of step 0 would not order step 0's inputs before it starts.
        stage0.copy_(packed[0][0], non_blocking=True)
        for i in range(n):
            if i % 2 == 0 and i + 1 < n:
                j = i + 1  # steps j and j + 1 (replicas j % R and j % R + 1 in host_cat)
                cnt = 2 if j + 1 < n else 1
                src = host_cat[(j % R) * nbytes:(j % R + cnt) * nbytes]
                K.stage_copy(pair_slots[((j - 1) // 2) % 3][:cnt * nbytes], src)
            dq, dk, dv, dpos, dsl, dslot, dbt = staged_for(i)
            K.paged_decode_step(dq, dk, dv, dpos, dslot, inv, pools[i % R], dbt, dsl,
                                out=douts[i], workspace=ws)
            b = i % 2
            k_done[b].record(comp)
            s_d2h.wait_event(k_done[b])
            with torch.cuda.stream(s_d2h):
                houts[b].copy_(douts[i], non_blocking=True)
        comp.wait_stream(s_d2h)
        if last is not None:
            last.record(comp)

    # All e2e steps in ONE CUDA graph with their copies, bracketed by
    # event-record nodes.
    with torch.cuda.stream(side):
        run_pipeline(min(e2e_steps, R))
    torch.cuda.synchronize(dev)
    ev_e2e = (torch.cuda.Event(enable_timing=True, external=True),
              torch.cuda.Event(enable_timing=True, external=True))
    g_e2e = capture([lambda: run_pipeline(e2e_steps, *ev_e2e)])
    g_e2e_warm = capture([lambda: run_pipeline(min(e2e_steps, max(args.warmup, 2)))])
    torch.cuda.synchronize(dev)
    # The pipeline computes the same outputs as the device-resident step.
    last_i = e2e_steps - 1
    K.paged_decode_step(qs[last_i % R], k, v, pos, slots[last_i % R], inv, pools[last_i % R],
                        bts[last_i % R], sl, out=outs[0], workspace=ws)
    torch.cuda.synchronize(dev)
    g_e2e.replay()
    torch.cuda.synchronize(dev)
    if not torch.equal(houts[last_i % 2], outs[0].cpu()):
        raise RuntimeError("pipelined end-to-end output differs from the device-resident step")
    g_e2e_warm.replay()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    g_e2e.replay()
    e3.record()
    torch.cuda.synchronize(dev)
    barrier()
    t_e2e = max_over_ranks(ev_e2e[0].elapsed_time(ev_e2e[1]) * 1e-3)
    t_e2e_replay = max_over_ranks(e2.elapsed_time(e3) * 1e-3)
    h2d_bytes = sum(sizes)
    d2h = houts[0].numel() * houts[0].element_size()
    err = K.error_word(dev)
    if err:
        raise RuntimeError(f"device error word {err} after the timed regions")

    if rank == 0:
        peak, peak_kind = measured_peaks()
        # The timed step is one launch of the fused decode-step kernel, so the
        # roofline is that launch: step time / step, bytes of the fused step.
        ab = alg_bytes(cfg, ctx, pages, fused=True)
        t_launch = t_step / args.steps
        achieved = ab / t_launch / 1e9
        ab_attn = alg_bytes(cfg, ctx, pages)
        line = {
            "metric": "decode tokens/s", "value": world * B * args.steps / t_step,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_step / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if dt == "bfloat16" else "f16",
            "data": "synthetic (seeded N(0,1) q/k/v/pool; seeded ragged contexts)",
            "config": decode_config(cfg, ctx, world),
            "method": {
                "l2": f"inputs larger than L2: {R} pool/table replicas rotated "
                      f"({R} x {ab / 1e6:.0f} MB touched per cycle)",
                "timing": f"one CUDA graph of the {args.steps} timed steps (PDL-chained) "
                          "between two event-record nodes, max over ranks",
                "replay_us_incl_submission": t_replay * 1e6,
            },
            "e2e": {"value": world * B * e2e_steps / t_e2e, "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "api": "vllm_mps_b200.kernels.stage_copy (packed pinned inputs -> device, "
                           "a PDL-chained copy kernel) + kernels.paged_decode_step, then one "
                           "copy-engine D2H of the output on a copy stream; all steps in one "
                           "CUDA graph between two event-record nodes",
                    "replay_us_incl_submission": t_e2e_replay * 1e6},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profile_traffic(cfg_name),
                         "peak_kind": peak_kind,
                         "kernel": "paged_decode_kernel (fused decode step)",
                         "kernel_us": t_launch * 1e6, "alg_bytes_per_launch": ab,
                         "attention_only": {"kernel_us": t_kernel * 1e6,
                                            "alg_bytes_per_launch": ab_attn,
                                            "achieved": ab_attn / t_kernel / 1e9,
                                            "frac": ab_attn / t_kernel / 1e9 / peak}},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps,
        }
        if world == 1 and not args.no_cpu_baseline and cpu_base:
            line["cpu_baseline"] = cpu_baseline(cfg, ctx, tables)
        return line
    return None


# ── prefill (kernel 3) ───────────────────────────────────────────────────────

PREFILL = {
    # Llama-3-8B attention shape (config 2), bf16: 16 prompts of 2048 tokens, no cached prefix.
    "prefill": (16, 2048, 32, 8, 128, "bfloat16", 500000.0,
                "Causal paged prefill, Llama-3-8B attention shape: 16 prompts x 2048 tokens, "
                "32 q / 8 kv heads, head_dim 128, bf16, block_size 16, permuted pool"),
    # TinyLlama attention shape (configs 0 and 4), fp16.
    "prefill_tinyllama": (16, 2048, 32, 4, 64, "float16", 10000.0,
                          "Causal paged prefill, TinyLlama attention shape: 16 prompts x 2048 "
                          "tokens, 32 q / 4 kv heads, head_dim 64, fp16, block_size 16, permuted pool"),
}


def prefill_flops(B, L, n_q, D):
    """QK^T and PV over the causal pairs: 4 * n_q * D per (row, key), L(L+1)/2 pairs per prompt."""
    return B * (L * (L + 1) // 2) * 4 * n_q * D


def prefill_cpu_baseline(B, L, n_q, n_kv, D, dt, theta, budget_s=10.0):
    """C oracle on sampled prompt rows (the reference computes a prompt token by token).

    Rows are taken at evenly spaced positions of one prompt, so their mean
    cost is the mean cost of a prompt row; tokens/s = rows / time.
    """
    from oracle import c_oracle
    from oracle.paged_attention_oracle import f32_to_bits, rope_inv_freq

    c_oracle.build()
    pages = (L + BLOCK - 1) // BLOCK
    rng = np.random.default_rng(7)
    pool = f32_to_bits(rng.standard_normal((pages, 2, BLOCK, n_kv, D), dtype=np.float32), dt)
    table = np.arange(pages, dtype=np.int32)[None, :]
    inv = rope_inv_freq(D, theta)
    threads = os.cpu_count() or 1
    q = f32_to_bits(rng.standard_normal((1, n_q, D), dtype=np.float32), dt)
    k = f32_to_bits(rng.standard_normal((1, n_kv, D), dtype=np.float32), dt)
    v = f32_to_bits(rng.standard_normal((1, n_kv, D), dtype=np.float32), dt)
    order = np.random.default_rng(8).permutation(L)
    c_oracle.decode_step(q, k, v, np.array([0]), np.array([1]), table, pool, inv, dt,
                         threads=threads)
    t0 = time.perf_counter()
    n = 0
    while n < L:
        pos = int(order[n])
        c_oracle.decode_step(q, k, v, np.array([pos]), np.array([pos + 1]), table, pool, inv,
                             dt, threads=threads)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    el = time.perf_counter() - t0
    return {"value": n / el, "unit": "tokens/s", "cores": c_oracle.max_threads(), "kind": "port",
            "sample": f"{n} rows at random positions of one {L}-token prompt in {el:.1f} s "
                      f"(token-by-token, as the reference prefills), C oracle, OpenMP"}


def run_prefill_reference(args, rank, world):
    B, L, n_q, n_kv, D, dtn, theta, desc = PREFILL[args.config]
    if True:
        if rank != 0:
            return 0
        base = prefill_cpu_baseline(B, L, n_q, n_kv, D, dtn, theta,
                                    budget_s=max(3.0, 2.0 * (args.steps + args.warmup)))
        v = base["value"]
        print(json.dumps({
            "metric": "prefill tokens/s", "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": B * L / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": desc, "global_batch": B, "parallelism": "host cores"},
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return 0


# A timed region at least this long runs under the power cap like the
# driver's seconds-long sustained GEMM loop, so it is measured against that.
SUSTAINED_AFTER_S = 0.5


def tensor_peak(timed_s):
    """(peak TFLOP/s, kind, (other peak, its name) or None) for a tensor-bound
    kernel whose timed region lasted ``timed_s`` seconds: the measured burst
    bf16 figure for a short region, the measured sustained one for a region
    of SUSTAINED_AFTER_S or longer."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        burst = float(m["bf16_tflops"])
        sustained = float(m.get("bf16_tflops_sustained") or 0.0)
    except Exception:
        return 1590.0, "fallback", None
    if sustained > 0 and timed_s >= SUSTAINED_AFTER_S:
        return sustained, f"measured (sustained: {timed_s:.2f} s timed)", (burst, "burst")
    return burst, f"measured (burst: {timed_s:.3f} s timed)", (
        (sustained, "sustained") if sustained > 0 else None)


def prefill_leg(args, cfg_name, rank, world, local_rank, cpu_base=True):
    """Kernel 3 on a PREFILL config: the record on rank 0, None elsewhere."""
    import torch

    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    B, L, n_q, n_kv, D, dtn, theta, desc = PREFILL[cfg_name]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dt = getattr(torch, dtn)
    pages = (L + BLOCK - 1) // BLOCK
    nb = B * pages + 64
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    pool = torch.randn((nb, 2, BLOCK, n_kv, D), generator=g, device=dev, dtype=torch.float32).to(dt)
    perm = torch.randperm(nb, device="cpu", generator=torch.Generator().manual_seed(rank))
    bt = perm[: B * pages].view(B, pages).to(torch.int32).to(dev)
    rows = B * L
    q = torch.randn((rows, n_q, D), generator=g, device=dev, dtype=torch.float32).to(dt)
    k = torch.randn((rows, n_kv, D), generator=g, device=dev, dtype=torch.float32).to(dt)
    v = torch.randn((rows, n_kv, D), generator=g, device=dev, dtype=torch.float32).to(dt)
    q_start = torch.zeros(B, dtype=torch.int32, device=dev)
    q_lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    cu = torch.arange(0, rows, L, dtype=torch.int32, device=dev)
    pos = torch.arange(L, dtype=torch.int32, device=dev).repeat(B)
    seq = torch.arange(B, device=dev).repeat_interleave(L)
    slots = (bt[seq, (pos // BLOCK).long()] * BLOCK + pos % BLOCK).to(torch.int32)
    inv = rope_inv_freq(D, theta).to(dev)
    out = torch.empty((rows, n_q, D), dtype=dt, device=dev)
    q_rot = q.clone()
    K.rope_reshape_and_cache(q, k, v, pos, slots, inv, pool, q_out=q_rot)

    def attn():
        K.paged_prefill_attention(q_rot, pool, bt, q_start, q_lens, cu, L, out=out)

    for _ in range(args.warmup):
        attn()
    torch.cuda.synchronize(dev)
    if K.error_word(dev):
        raise RuntimeError("device error word set during warm-up")
    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        e0.record()
        for _ in range(args.steps):
            attn()
        e1.record()
        torch.cuda.synchronize(dev)
    barrier()
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3)

    # End to end through the public API: host q/k/v in pinned memory, kernel 1
    # (RoPE + K/V write) and kernel 3, output copied back, every step.
    hq, hk, hv = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    hout = torch.empty_like(out, device="cpu").pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def e2e():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        K.rope_reshape_and_cache(dq, dk, dv, pos, slots, inv, pool)
        K.paged_prefill_attention(dq, pool, bt, q_start, q_lens, cu, L, out=out)
        hout.copy_(out, non_blocking=True)

    e2e_steps = max(3, args.steps // 4)
    for _ in range(3):
        e2e()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(e2e_steps):
        e2e()
    e3.record()
    torch.cuda.synchronize(dev)
    barrier()
    t_e2e = max_over_ranks(e2.elapsed_time(e3) * 1e-3)
    if K.error_word(dev):
        raise RuntimeError("device error word set during the timed region")
    if rank == 0:
        peak, kind, other = tensor_peak(t)
        flops = prefill_flops(B, L, n_q, D)
        achieved = flops / (t / args.steps) / 1e12
        line = {
            "metric": "prefill tokens/s", "value": world * rows * args.steps / t,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if dt == torch.bfloat16 else "f16",
            "data": "synthetic (seeded N(0,1) q/k/v/pool)",
            "config": {"workload": desc, "global_batch": B * world, "seq_len": L,
                       "parallelism": f"sequence-sharded x{world}",
                       "l2": f"inputs larger than L2 (q {rows * n_q * D * 2 / 1e6:.0f} MB, out the "
                             f"same, K/V {B * L * n_kv * D * 4 / 1e6:.0f} MB per rank)",
                       "timing": "back-to-back launches, CUDA events, max over ranks"},
            "e2e": {"value": world * rows * e2e_steps / t_e2e, "unit": "tokens/s",
                    "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in (hq, hk, hv)),
                    "d2h_bytes_per_step": hout.numel() * hout.element_size(),
                    "api": "kernels.rope_reshape_and_cache + kernels.paged_prefill_attention, "
                           "pinned host q/k/v"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None, "peak_kind": kind,
                         "timed_s": t,
                         **({f"frac_vs_{other[1]}": achieved / other[0]} if other else {}),
                         "kernel": "paged_prefill_kernel",
                         "kernel_us": t / args.steps * 1e6, "alg_flops_per_launch": flops},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps,
        }
        if world == 1 and not args.no_cpu_baseline and cpu_base:
            line["cpu_baseline"] = prefill_cpu_baseline(B, L, n_q, n_kv, D, dtn, theta)
        return line
    return None


# ── engine decode (configs 0 and 2) ─────────────────────────────────────────

ENGINE = {
    # name: (layers, hidden, q heads, kv heads, mlp, vocab, theta, dtype, batch,
    #        prompt lo, prompt hi, decode steps, description)
    "c0": (22, 2048, 32, 4, 5632, 32000, 10000.0, "float16", 8, 32, 32, 20,
           "Config 0: TinyLlama-1.1B shape, random fp16 weights (seed 0), 8 prompts x 32 ids, "
           "20 greedy decode steps, physical mode (per-layer pools, kernel-3 prefill)"),
    "c2": (32, 4096, 32, 8, 14336, 128256, 500000.0, "bfloat16", 256, 128, 4096, 128,
           "Config 2: Llama-3-8B shape, random bf16 weights, 256 prompts U[128,4096], "
           "128 greedy decode steps, physical mode (per-layer pools, kernel-3 prefill)"),
}


def run_engine(args, rank, world, local_rank):
    """Engine decode throughput: generated tokens per second of decode steps.

    Every rank runs its own engine on its own requests (sequence sharding,
    weak scaling).  The timed region is the decode steps after the first
    step (which also prefills every prompt), each one the engine's public
    ``step()``: host token ids in, metadata built and copied, one CUDA-graph
    replay (22/32 layers, each with the fused decode-step kernel and the fused
    residual/RMSNorm/SiLU kernels between cuBLAS GEMMs), greedy sampling,
    host token ids out.
    """
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.engine.llm_engine import LLMEngine

    (nl, hid, nh, nkv, mlp, vocab, theta, dtn, B, plo, phi, steps, desc) = ENGINE[args.config]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dt = getattr(torch, dtn)
    cfg = LlamaConfig(hidden_size=hid, intermediate_size=mlp, num_hidden_layers=nl,
                      num_attention_heads=nh, num_key_value_heads=nkv, vocab_size=vocab,
                      rms_norm_eps=1e-5, rope_theta=theta, max_position_embeddings=8192,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(dt).eval()
    rng = np.random.default_rng(100 + rank)
    lens = rng.integers(plo, phi + 1, size=B)
    prompts = [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]
    steps = min(steps, args.steps) if args.steps < steps else steps
    blocks = int(sum((int(n) + steps + 16) // 16 + 1 for n in lens)) + 16
    eng = LLMEngine.from_model(model, num_gpu_blocks=blocks, num_cpu_blocks=16, max_batch_size=B,
                               max_tokens_per_step=10 ** 9, mode="physical", dtype=dt, device=dev,
                               max_prefill_rows=16384, pipeline=not args.sync_engine)
    eng.capture_decode_graphs()  # startup work, outside the timed region
    for p in prompts:
        eng.add_request(p, SamplingParams(temperature=0.0, max_tokens=steps + 1))
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    eng.step()  # admits every request, prefills all prompts, first token
    torch.cuda.synchronize(dev)
    t_prefill = time.perf_counter() - t0
    for _ in range(min(args.warmup, 3)):
        eng.step()
    dist = None
    if world > 1:
        import torch.distributed as dist
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_timed, toks = steps - min(args.warmup, 3), 0
    with ClockSampler(dev.index or 0) as clocks:
        e0.record()
        for _ in range(n_timed):
            toks += len(eng.step())
        e1.record()
        torch.cuda.synchronize(dev)
    t = e0.elapsed_time(e1) * 1e-3
    if dist is not None:
        tt = torch.tensor([t, toks], dtype=torch.float64, device=dev)
        dist.all_reduce(tt[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tt[1:], op=dist.ReduceOp.SUM)
        t, toks = float(tt[0]), int(tt[1])
    from vllm_mps_b200 import kernels as K

    if K.error_word(dev):
        raise RuntimeError("device error word set during the engine run")
    if rank == 0:
        peak, peak_kind = measured_peaks()
        n_params = sum(p.numel() for p in model.parameters())
        ctx_mean = float(lens.mean()) + 3 + n_timed / 2
        kv_bytes = B * ctx_mean * nl * nkv * (hid // nh) * 2 * 2
        step_bytes = n_params * 2 + kv_bytes  # weights once + every layer's K/V history
        t_step = t / n_timed
        line = {
            "metric": "decode tokens/s", "value": toks / t, "unit": "tokens/s", "n_gpus": world,
            "steps": n_timed, "warmup": min(args.warmup, 3) + 1, "ms_per_step": t_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if dt == torch.bfloat16 else "f16",
            "data": "synthetic (random-init weights, seeded random prompt ids)",
            "config": {"workload": desc, "global_batch": B * world,
                       "seq_len": f"prompts U[{plo},{phi}] + {steps} generated",
                       "parallelism": f"sequence-sharded x{world}",
                       "prefill_s_first_step": t_prefill,
                       "engine_loop": "synchronous" if args.sync_engine else "pipelined",
                       "timing": "CUDA events around the engine's step() calls"},
            "e2e": {"value": toks / t, "unit": "tokens/s",
                    "h2d_bytes_per_step": B * 8 + B * (int(ctx_mean) // 16 + 4) * 4,
                    "d2h_bytes_per_step": B * 8,
                    "api": "LLMEngine.step(): host token ids in, host token ids out "
                           "(pipelined: each call returns the previous launch's ids)"},
            "roofline": {"bound": "hbm", "achieved": step_bytes / t_step / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": step_bytes / t_step / 1e9 / peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole decode step (weights + every layer's K/V history)",
                         "alg_bytes_per_step": step_bytes},
            "clocks": clocks.summary(),
            # Per step: the decode-step kernel, two add_rmsnorm per layer and
            # the first input norm, and at decode batch sizes the decode GEMMs
            # (QKV, O, [gate|up] with SiLU * up, down, LM head); else cuBLAS
            # GEMMs and a silu_mul per layer.
            "gpu_launches": n_timed * (eng._graphs.own_kernels_per_step(B) if eng._graphs
                                       else nl),
            "cpu_baseline": None,
            "cpu_baseline_note": "the reference's engine is Python on its CPU path; config 0 "
                                 "took 33 tokens/s on 8 host cores in the survey (config 2 is "
                                 "impractical on CPU); the kernel-level port baselines are the "
                                 "c1/c3/prefill lines",
        }
        print(json.dumps(line), flush=True)
    return 0


# ── config 4: mixed prefill + decode, sequence-sharded ───────────────────────

C4 = ("Config 4: TinyLlama shape (config 0 model), 1024 requests, prompts "
      "clip(round(lognormal(6,1)),16,4096), outputs U[16,512], FCFS, preemption when the pool "
      "is 90% full, sequence-sharded (one engine per GPU, NCCL token gather every 16 steps)")


def c4_leg(args, rank, world, local_rank, n_req=1024):
    """All config-4 requests to completion through the sequence-sharded engine.

    Every rank runs ``ShardedEngine`` over its own ``LLMEngine`` (at N = 1 the
    same loop, without the collective); the ranks exchange their sampled
    tokens with one NCCL ``all_gather_into_tensor`` every 16 steps.  Returns
    the record on rank 0 (None elsewhere): generated tokens/s of the whole
    job, steps, gathers, per-rank time in local steps and in the gathers.
    """
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.engine.distributed import ShardedEngine
    from vllm_mps_b200.engine.llm_engine import LLMEngine

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    nl, hid, nh, nkv, mlp, vocab, theta, dtn = ENGINE["c0"][:8]
    cfg = LlamaConfig(hidden_size=hid, intermediate_size=mlp, num_hidden_layers=nl,
                      num_attention_heads=nh, num_key_value_heads=nkv, vocab_size=vocab,
                      rms_norm_eps=1e-5, rope_theta=theta, max_position_embeddings=8192,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.float16).eval()
    rng = np.random.default_rng(4)
    p_lens = np.clip(np.round(rng.lognormal(6, 1, n_req)), 16, 4096).astype(int)
    o_lens = rng.integers(16, 513, n_req)
    prompts = [rng.integers(0, vocab, size=int(n)).tolist() for n in p_lens]
    params = [SamplingParams(temperature=0.0, max_tokens=int(m)) for m in o_lens]
    eng = LLMEngine.from_model(model, num_gpu_blocks=16384, num_cpu_blocks=4096,
                               max_batch_size=256, max_tokens_per_step=10 ** 9, mode="physical",
                               preempt_watermark=0.9, dtype=torch.float16, device=dev,
                               max_prefill_rows=16384, pipeline=not args.sync_engine)
    dist = None
    if world > 1:
        import torch.distributed as dist
    eng.capture_decode_graphs()  # startup work: every batch bucket up to 256
    eng.warm_prefill_gemms()     # startup work: every padded prefill GEMM row count
    # Warm-up through this rank's engine, untimed: 64 requests of the same
    # length distribution (other seeded ids) with short outputs, so that the
    # prefill chunk shapes, batch buckets, workspaces and the allocator's
    # blocks of the timed run are set up before it, plus one full 16384-row
    # prefill chunk.
    wrng = np.random.default_rng(5)
    for n in np.clip(np.round(wrng.lognormal(6, 1, 64)), 16, 4096).astype(int):
        eng.add_request(wrng.integers(0, vocab, size=int(n)).tolist(),
                        SamplingParams(temperature=0.0, max_tokens=16))
    for i in range(4):
        eng.add_request(wrng.integers(0, vocab, size=4097).tolist(),
                        SamplingParams(temperature=0.0, max_tokens=2))
    while not eng.is_finished():
        eng.step()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    with ClockSampler(dev.index or 0) as clocks:
        e0.record()
        if dist is not None:
            sharded = ShardedEngine(eng, gather_every=16)
            sharded.add_requests(prompts, params)
            outs = sharded.run()
            done = sum(len(o.token_ids) for o in outs.values())
            steps, gathers = sharded.steps, sharded.gathers
            step_s, gather_s = sharded.step_seconds, sharded.gather_seconds
        else:
            start_tokens = eng.total_tokens_generated
            for p, sp in zip(prompts, params):
                eng.add_request(p, sp)
            steps = 0
            t_s = time.perf_counter()
            while not eng.is_finished():
                eng.step()
                steps += 1
            step_s, gather_s, gathers = time.perf_counter() - t_s, 0.0, 0
            done = eng.total_tokens_generated - start_tokens
        e1.record()
        torch.cuda.synchronize(dev)
    t = e0.elapsed_time(e1) * 1e-3
    per_rank = np.array([[t, step_s, gather_s, steps]], dtype=np.float64)
    if dist is not None:
        mine = torch.tensor(per_rank[0], dtype=torch.float64, device=dev)
        allr = torch.empty(world * 4, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(allr, mine)
        per_rank = allr.view(world, 4).cpu().numpy()
        t = float(per_rank[:, 0].max())
    from vllm_mps_b200 import kernels as K

    if K.error_word(dev):
        raise RuntimeError("device error word set during the config-4 run")
    if done != int(o_lens.sum()):
        raise RuntimeError(f"generated {done} tokens, expected {int(o_lens.sum())}")
    if rank != 0:
        return None
    return {
        "metric": "generated tokens/s (mixed prefill + decode)", "value": done / t,
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "gathers": gathers,
        "ms_per_step": t / max(steps, 1) * 1e3, "higher_is_better": True,
        "scaling": "strong", "dtype": "f16",
        "data": "synthetic (random-init weights, seeded lognormal prompts)",
        "config": {"workload": C4 if n_req == 1024 else f"{C4} [first {n_req} requests]",
                   "global_batch": n_req, "parallelism": f"sequence-sharded x{world}",
                   "engine_loop": "synchronous" if args.sync_engine else "pipelined",
                   "prompt_tokens": int(p_lens.sum()), "generated_tokens": int(o_lens.sum()),
                   "timing": "CUDA events around the whole run, max over ranks"},
        "per_rank": {"run_s": per_rank[:, 0].round(4).tolist(),
                     "local_step_s": per_rank[:, 1].round(4).tolist(),
                     "gather_s": per_rank[:, 2].round(4).tolist(),
                     "gather_share": (per_rank[:, 2] / np.maximum(per_rank[:, 0], 1e-9))
                     .round(4).tolist()},
        "wall_s": time.perf_counter() - t_wall,
        "preempted_final": eng.scheduler.get_num_preempted(),
        "e2e": {"value": done / t, "unit": "tokens/s", "h2d_bytes_per_step": None,
                "d2h_bytes_per_step": None,
                "api": "LLMEngine / ShardedEngine: host token ids in and out"},
        "clocks": clocks.summary(),
    }


def run_c4(args, rank, world, local_rank):
    line = c4_leg(args, rank, world, local_rank)
    if line is not None:
        line.update({"warmup": 1, "vs_baseline": None, "roofline": None, "gpu_launches": None,
                     "cpu_baseline": None})
        print(json.dumps(line), flush=True)
    return 0


# ── decode GEMM (the engine's projections at decode batch sizes) ───────────

GEMM_SHAPES = (
    # name, output features, K, gated ([gate; up] weight of 2N rows + SiLU * up)
    ("qkv", 2560, 2048, False),
    ("o", 2048, 2048, False),
    ("gate_up", 5632, 2048, True),
    ("down", 2048, 5632, False),
    ("lm_head", 32000, 2048, False),
)


def run_gemm(args, rank, world, local_rank):
    """Decode GEMM on the TinyLlama decode projections (M = 8, fp16).

    A step is one pass of the five projections of a config-0 decode step
    (QKV, O, [gate; up] with SiLU * up, down, LM head) through
    ``kernels.decode_gemm``; four weight sets (876 MB) rotate so inputs are
    larger than L2.  ``value`` is weight GB/s over the step; each projection
    is also timed alone (40 launches in a CUDA graph) next to cuBLAS
    (``F.linear``, plus ``silu_mul`` for the gated one).
    """
    import torch
    import torch.nn.functional as F

    from vllm_mps_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M, R, dt = 8, 4, torch.float16
    g = torch.Generator(device=dev).manual_seed(5)
    W = {n: [(torch.randn((2 * N if gated else N), Kd, generator=g, device=dev) / Kd ** 0.5).to(dt)
             for _ in range(R)] for n, N, Kd, gated in GEMM_SHAPES}
    X = {Kd: torch.randn(M, Kd, generator=g, device=dev).to(dt) for Kd in (2048, 5632)}
    OUT = {n: torch.empty(M, N, device=dev, dtype=dt) for n, N, Kd, gated in GEMM_SHAPES}
    weight_bytes = sum(W[n][0].numel() * 2 for n, *_ in GEMM_SHAPES)

    def step(r):
        for n, N, Kd, gated in GEMM_SHAPES:
            K.decode_gemm(X[Kd], W[n][r], out=OUT[n], silu_mul=gated)

    def capture(fns):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for f in fns:
                f()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for f in fns:
                f()
        return gr

    def timed(gr, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e-3

    g_steps = capture([lambda r=r: step(r) for r in range(R)])
    for _ in range(max(1, args.warmup // R)):
        g_steps.replay()
    reps = max(1, args.steps // R)
    with ClockSampler(dev.index or 0) as clocks:
        t = timed(g_steps, reps)
    n_steps = reps * R
    t_step = t / n_steps

    per = {}
    for n, N, Kd, gated in GEMM_SHAPES:
        it = [0]

        def ours(n=n, Kd=Kd, gated=gated):
            it[0] = (it[0] + 1) % R
            K.decode_gemm(X[Kd], W[n][it[0]], out=OUT[n], silu_mul=gated)

        def cublas(n=n, Kd=Kd, gated=gated):
            it[0] = (it[0] + 1) % R
            y = F.linear(X[Kd], W[n][it[0]])
            if gated:
                K.silu_mul(y, out=OUT[n])

        a, b = capture([ours] * 40), capture([cublas] * 40)
        timed(a, 2), timed(b, 2)
        ta, tb = timed(a, 5) / 200, timed(b, 5) / 200
        per[n] = {"us": round(ta * 1e6, 2), "gb_s": round(W[n][0].numel() * 2 / ta / 1e9, 1),
                  "cublas_us": round(tb * 1e6, 2)}

    # End to end: X from pinned host memory in, the LM-head logits back, per step.
    xh = {Kd: X[Kd].cpu().pin_memory() for Kd in X}
    oh = torch.empty(M, 32000, dtype=dt).pin_memory()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = min(n_steps, 200)
    e0.record()
    for i in range(n_e2e):
        for Kd in X:
            X[Kd].copy_(xh[Kd], non_blocking=True)
        step(i % R)
        oh.copy_(OUT["lm_head"], non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    t_e2e = e0.elapsed_time(e1) * 1e-3 / n_e2e
    if K.error_word(dev):
        raise RuntimeError("device error word set during the decode-GEMM run")

    if rank == 0:
        peak, peak_kind = measured_peaks()
        lm = per["lm_head"]
        traffic = None
        try:
            for line in open(os.path.join(ROOT, "profiles", "decode_gemm_tinyllama.md")):
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":")[1])
        except OSError:
            pass
        # CPU baseline: the same five projections as torch float32 matmuls on
        # the host cores (the reference runs them as nn.Linear on its CPU path).
        torch.set_num_threads(os.cpu_count() or 1)
        wc = {n: W[n][0].float().cpu() for n, *_ in GEMM_SHAPES}
        xc = {Kd: X[Kd].float().cpu() for Kd in X}
        t0, n_cpu = time.perf_counter(), 0
        while time.perf_counter() - t0 < 5.0 and n_cpu < 50:
            for n, N, Kd, gated in GEMM_SHAPES:
                y = xc[Kd] @ wc[n].t()
                if gated:
                    y = F.silu(y[:, :N]) * y[:, N:]
            n_cpu += 1
        t_cpu = (time.perf_counter() - t0) / n_cpu
        line = {
            "metric": "decode-GEMM weight stream", "value": weight_bytes / t_step / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": n_steps, "warmup": args.warmup,
            "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1)/sqrt(K) weights, N(0,1) activations)",
            "config": {"workload": "TinyLlama decode projections at M=8 (QKV, O, [gate;up] + "
                                   "SiLU*up, down, LM head) through kernels.decode_gemm",
                       "global_batch": M, "weight_bytes_per_step": weight_bytes,
                       "l2": "inputs larger than L2: 4 weight sets (876 MB) rotated",
                       "per_projection": per},
            "e2e": {"value": weight_bytes / t_e2e / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": sum(x.numel() * 2 for x in X.values()),
                    "d2h_bytes_per_step": oh.numel() * 2,
                    "api": "kernels.decode_gemm; per step X copied in from pinned memory and "
                           "the LM-head output copied back, not overlapped"},
            "roofline": {"bound": "hbm", "achieved": lm["gb_s"], "peak": peak, "unit": "GB/s",
                         "frac": lm["gb_s"] / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "decode_gemm_kernel (LM head, 32000 x 2048, M=8)",
                         "kernel_us": lm["us"], "alg_bytes_per_launch": 32000 * 2048 * 2},
            "clocks": clocks.summary(),
            "gpu_launches": n_steps * len(GEMM_SHAPES),
            "cpu_baseline": {"value": weight_bytes / t_cpu / 1e9, "unit": "GB/s",
                             "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{n_cpu} passes of the five projections, torch float32 "
                                       "matmul on the host cores"},
        }
        print(json.dumps(line), flush=True)
    return 0


BGEMM_SHAPES = (
    # name, M (batch), N (output features), K -- Llama-3-8B projections at the config-2 batch
    ("qkv", 256, 6144, 4096),
    ("o", 256, 4096, 4096),
    ("gate_up", 256, 28672, 4096),
    ("down", 256, 4096, 14336),
)


def run_bgemm(args, rank, world, local_rank):
    """Kernel 5 (``kernels.batch_gemm``: tcgen05, cluster split-K) on the batch-256
    projections of a Llama-3-8B decode step, next to cuBLAS (``torch.matmul``).

    A step is one pass of the four projections; four weight sets (1.75 GB)
    rotate so inputs are larger than L2.  Each projection is also timed alone
    (40 launches in a CUDA graph) beside cuBLAS on the same inputs.
    """
    import torch

    from vllm_mps_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    R, dt = 4, torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(7)
    W = {n: [(torch.randn(N, Kd, generator=g, device=dev) / Kd ** 0.5).to(dt) for _ in range(R)]
         for n, M, N, Kd in BGEMM_SHAPES}
    X = {n: (torch.randn(M, Kd, generator=g, device=dev) * 0.5).to(dt) for n, M, N, Kd in BGEMM_SHAPES}
    OUT = {n: torch.empty(M, N, device=dev, dtype=dt) for n, M, N, Kd in BGEMM_SHAPES}
    flops = sum(2 * M * N * Kd for _, M, N, Kd in BGEMM_SHAPES)
    wbytes = sum(N * Kd * 2 for _, M, N, Kd in BGEMM_SHAPES)

    def capture(fns):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for f in fns:
                f()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for f in fns:
                f()
        return gr

    def timed(gr, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e-3

    # One split-K workspace per projection, allocated before any capture.
    WS = {n: torch.empty(max(16, K.batch_gemm_workspace_bytes(M, N, Kd, X[n].dtype)),
                         dtype=torch.uint8, device=dev)
          for n, M, N, Kd in BGEMM_SHAPES}

    def step(r):
        for n, *_ in BGEMM_SHAPES:
            K.batch_gemm(X[n], W[n][r], out=OUT[n], workspace=WS[n])

    g_steps = capture([lambda r=r: step(r) for r in range(R)])
    for _ in range(max(1, args.warmup // R)):
        g_steps.replay()
    reps = max(1, args.steps // R)
    with ClockSampler(dev.index or 0) as clocks:
        t = timed(g_steps, reps)
    n_steps = reps * R
    t_step = t / n_steps
    per = {}
    for n, M, N, Kd in BGEMM_SHAPES:
        it = [0]

        def ours(n=n):
            it[0] = (it[0] + 1) % R
            K.batch_gemm(X[n], W[n][it[0]], out=OUT[n], workspace=WS[n])

        def cublas(n=n):
            it[0] = (it[0] + 1) % R
            torch.matmul(X[n], W[n][it[0]].t(), out=OUT[n])

        a, b = capture([ours] * 40), capture([cublas] * 40)
        timed(a, 2), timed(b, 2)
        ta, tb = timed(a, 5) / 200, timed(b, 5) / 200
        per[n] = {"M": M, "N": N, "K": Kd, "split": K.batch_gemm_split(M, N, Kd),
                  "us": round(ta * 1e6, 2), "tflops": round(2 * M * N * Kd / ta / 1e12, 1),
                  "cublas_us": round(tb * 1e6, 2)}
    # End to end: every step's X in from pinned host memory, the outputs back.
    xh = {n: X[n].cpu().pin_memory() for n in X}
    oh = {n: torch.empty(OUT[n].shape, dtype=dt).pin_memory() for n in OUT}
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = min(n_steps, 100)
    e0.record()
    for i in range(n_e2e):
        for n in X:
            X[n].copy_(xh[n], non_blocking=True)
        step(i % R)
        for n in OUT:
            oh[n].copy_(OUT[n], non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    t_e2e = e0.elapsed_time(e1) * 1e-3 / n_e2e
    if K.error_word(dev):
        raise RuntimeError("device error word set during the batch-GEMM run")
    if rank == 0:
        import torch as _t

        _t.set_num_threads(os.cpu_count() or 1)
        wc = {n: W[n][0][:1024].float().cpu() for n in W}  # a bounded sample: 1024 rows each
        xc = {n: X[n].float().cpu() for n in X}
        t0, n_cpu = time.perf_counter(), 0
        while time.perf_counter() - t0 < 5.0 and n_cpu < 20:
            for n in W:
                xc[n] @ wc[n].t()
            n_cpu += 1
        t_cpu = (time.perf_counter() - t0) / n_cpu
        cpu_flops = sum(2 * X[n].shape[0] * 1024 * X[n].shape[1] for n in W)
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peak = (float(json.load(f)["bf16_tflops"]), "measured (burst)")
        except Exception:
            peak = (1590.0, "fallback")
        achieved = flops / t_step / 1e12
        line = {
            "metric": "batch-GEMM throughput", "value": achieved, "unit": "TFLOP/s", "n_gpus": 1,
            "steps": n_steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1)/sqrt(K) weights, N(0,0.25) activations)",
            "config": {"workload": "Llama-3-8B decode projections at batch 256 (QKV, O, [gate;up], "
                                   "down) through kernels.batch_gemm",
                       "global_batch": 256, "weight_bytes_per_step": wbytes,
                       "l2": "inputs larger than L2: 4 weight sets (1.75 GB) rotated",
                       "per_projection": per},
            "e2e": {"value": flops / t_e2e / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": sum(x.numel() * 2 for x in X.values()),
                    "d2h_bytes_per_step": sum(o.numel() * 2 for o in OUT.values()),
                    "api": "kernels.batch_gemm; per step X in from pinned memory, outputs back"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak[0],
                         "unit": "TFLOP/s", "frac": achieved / peak[0], "traffic": None,
                         "peak_kind": peak[1], "kernel": "batch_gemm_kernel (4 projections)",
                         "hbm_gb_s": wbytes / t_step / 1e9},
            "clocks": clocks.summary(),
            "gpu_launches": n_steps * len(BGEMM_SHAPES),
            "cpu_baseline": {"value": cpu_flops / t_cpu / 1e12, "unit": "TFLOP/s",
                             "cores": _t.get_num_threads(), "kind": "port",
                             "sample": f"{n_cpu} passes of the four projections on 1024 output "
                                       "features each, torch float32 matmul on the host cores"},
        }
        print(json.dumps(line), flush=True)
    return 0


def _summary(rec):
    """The keys of a leg's record that a sub-record keeps."""
    keep = ("metric", "value", "unit", "steps", "gathers", "ms_per_step", "scaling", "dtype",
            "roofline", "per_rank", "wall_s", "clocks")
    out = {k: rec[k] for k in keep if k in rec}
    out["workload"] = rec["config"]["workload"]
    if rec.get("e2e"):
        out["e2e"] = {k: rec["e2e"][k] for k in ("value", "unit") if k in rec["e2e"]}
    return out


def add_subrecords(args, line, rank, world, local_rank):
    """Run the other configs after the C1 headline; every rank takes part.

    * ``c3``: config 3 (4 x 131072, split-K) through the same fused step,
      HBM roofline of its launch;
    * ``prefill``: kernel 3 on the Llama-3-8B attention shape, tensor
      roofline against the measured bf16 peak (the sustained figure when
      the timed region lasts SUSTAINED_AFTER_S or longer, else the burst
      one; the other fraction is reported beside it);
    * ``engine_c4``: config 4 (1024 mixed requests) through the
      sequence-sharded engine with its NCCL token gather: generated tokens/s,
      steps, gathers and each rank's time in local steps and in the gathers.
    """
    import gc

    import torch

    subs = {}
    for name, fn in (("c3", lambda: decode_leg(args, "c3", rank, world, local_rank, cpu_base=False)),
                     ("prefill", lambda: prefill_leg(args, "prefill", rank, world, local_rank,
                                                     cpu_base=False)),
                     ("engine_c4", lambda: c4_leg(args, rank, world, local_rank))):
        gc.collect()
        torch.cuda.empty_cache()
        rec = fn()
        if rank == 0:
            subs[name] = _summary(rec)
    if rank == 0:
        line["subrecords"] = subs
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config",
                    choices=sorted(CONFIGS) + sorted(PREFILL) + sorted(ENGINE)
                    + ["c4", "gemm", "bgemm"],
                    default="c1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="c1: skip the c3 / prefill / sharded-engine sub-records")
    ap.add_argument("--sync-engine", action="store_true",
                    help="engine configs: the synchronous step loop instead of the pipelined one")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = CONFIGS.get(args.config)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and cfg is not None:
        return run_reference(args, cfg, rank, world)
    if args.impl == "reference" and (args.config in ENGINE or args.config in ("c4", "gemm", "bgemm")):
        why = ("the reference engine is Python on its CPU path and does not travel to the GPU box; "
               "see the c1/c3/prefill reference lines")
        if args.config in ("gemm", "bgemm"):
            why = ("the reference runs these projections as nn.Linear inside its CPU engine; the "
                   "ours-line's cpu_baseline times them as torch float32 matmuls on the host cores")
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}))
        return 0
    if args.impl == "reference":
        return run_prefill_reference(args, rank, world)
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config == "c4":
            return run_c4(args, rank, world, local_rank)
        if args.config == "gemm":
            return run_gemm(args, rank, world, local_rank)
        if args.config == "bgemm":
            return run_bgemm(args, rank, world, local_rank)
        if args.config in ENGINE:
            return run_engine(args, rank, world, local_rank)
        if cfg is None:
            line = prefill_leg(args, args.config, rank, world, local_rank)
        else:
            line = decode_leg(args, args.config, rank, world, local_rank)
            if args.config == "c1" and not args.no_subrecords:
                line = add_subrecords(args, line, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
