"""The PDL-chained stage copy (vmps_stage_copy) on the GPU.

It moves a decode step's inputs from pinned host memory into device memory
as one link of a chain of programmatically launched kernels.  Checked: the
bytes arrive exactly (host and device sources, sizes that are not a multiple
of the copy's unrolled stride), decode steps staged one launch ahead in a
CUDA graph read their staged inputs (same bits as the steps run on inputs
copied by the copy engine), and bad arguments are refused on the host.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [16, 4096, 361_000 // 16 * 16, (1 << 22) + 48])
def test_stage_copy_moves_exact_bytes(cuda_device, nbytes):
    from vllm_mps_b200 import kernels as K

    g = torch.Generator().manual_seed(nbytes)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g).pin_memory()
    dst = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    K.stage_copy(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), src)
    dst2 = torch.zeros_like(dst)
    K.stage_copy(dst2, dst)  # device source
    torch.cuda.synchronize()
    assert torch.equal(dst2, dst)


def _step_inputs(seed, B, n_q, n_kv, D, nb):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 400, B).astype(np.int32)
    pages = (ctx + 15) // 16
    perm = rng.permutation(nb)
    bt = np.zeros((B, 25), np.int32)
    off = 0
    for i, p in enumerate(pages):
        bt[i, :p] = perm[off:off + p]
        off += p
    pos = (ctx - 1).astype(np.int32)
    slots = np.array([bt[i, p // 16] * 16 + p % 16 for i, p in enumerate(pos)], np.int32)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, n_q, D, generator=g).half()
    k = torch.randn(B, n_kv, D, generator=g).half()
    v = torch.randn(B, n_kv, D, generator=g).half()
    return [q, k, v, torch.from_numpy(pos), torch.from_numpy(slots), torch.from_numpy(ctx),
            torch.from_numpy(bt)]


def test_stage_copy_feeds_graph_captured_decode_steps(cuda_device):
    """Two steps in a CUDA graph: step 0's inputs copied by the copy engine,
    step 1's staged from pinned host memory by the stage copy launched before
    step 0: the outputs and the pool are bit-identical to the same steps run
    eagerly on inputs copied by the copy engine."""
    from vllm_mps_b200 import kernels as K
    from vllm_mps_b200.layers.rotary_embedding import rope_inv_freq

    dev = cuda_device
    B, n_q, n_kv, D, nb = 16, 32, 4, 64, 512
    steps = [_step_inputs(s, B, n_q, n_kv, D, nb) for s in (0, 1)]
    shapes = [t.shape for t in steps[0]]
    dts = [t.dtype for t in steps[0]]

    def pack(parts):
        flat = [t.contiguous().view(torch.uint8).reshape(-1) for t in parts]
        offs, o = [], 0
        for t in flat:
            offs.append(o)
            o += (t.numel() + 255) // 256 * 256
        host = torch.zeros(o, dtype=torch.uint8).pin_memory()
        for t, off in zip(flat, offs):
            host[off:off + t.numel()].copy_(t)
        return host, offs, [t.numel() for t in flat]

    packed = [pack(p) for p in steps]
    offs, sizes = packed[0][1], packed[0][2]
    stage = [torch.empty(packed[0][0].numel(), dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(buf):
        return [buf[o:o + n].view(dt).view(sh) for o, n, dt, sh in zip(offs, sizes, dts, shapes)]

    inv = rope_inv_freq(D, 10000.0).to(dev)
    g = torch.Generator().manual_seed(9)
    pool0 = torch.randn(nb, 2, 16, n_kv, D, generator=g).half().to(dev)
    pool_ref, pool_g = pool0.clone(), pool0.clone()
    ws = K.DecodeWorkspace()
    refs = []
    for p in steps:
        q, k, v, pos, slots, ctx, bt = (t.to(dev) for t in p)
        refs.append(K.paged_decode_step(q, k, v, pos, slots, inv, pool_ref, bt, ctx, workspace=ws))
    torch.cuda.synchronize()
    outs = [torch.empty(B, n_q, D, dtype=torch.half, device=dev) for _ in range(2)]

    def run(pool):
        # Step 0 by copy engine (a full dependency), step 1 by stage copy one
        # launch ahead of the step that reads it.
        stage[0].copy_(packed[0][0], non_blocking=True)
        K.stage_copy(stage[1], packed[1][0])
        for s in range(2):
            q, k, v, pos, slots, ctx, bt = views(stage[s])
            K.paged_decode_step(q, k, v, pos, slots, inv, pool, bt, ctx, out=outs[s], workspace=ws)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        run(pool0.clone())  # warm-up outside the graph
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    for b in stage:
        b.zero_()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        run(pool_g)
    gr.replay()
    torch.cuda.synchronize()
    for s in range(2):
        assert torch.equal(outs[s], refs[s]), s
    assert torch.equal(pool_g.view(torch.int16), pool_ref.view(torch.int16))


def test_stage_copy_rejects_bad_arguments(cuda_device):
    from vllm_mps_b200 import kernels as K

    dst = torch.zeros(64, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError):
        K.stage_copy(dst, torch.zeros(64, dtype=torch.uint8))  # not pinned
    with pytest.raises(ValueError):
        K.stage_copy(dst, torch.zeros(48, dtype=torch.uint8).pin_memory())  # size differs
    with pytest.raises(ValueError):
        K.stage_copy(dst[:40], torch.zeros(40, dtype=torch.uint8).pin_memory())  # not 16-byte multiple
