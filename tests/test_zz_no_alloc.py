"""The allocation-free decode entry point, called through the C ABI.

``vmps_paged_decode_attention_noalloc`` is for callers that cannot allocate
device memory while they run (an FFI host with no caching allocator, or a
process that has reserved all free HBM for its KV pool up front): it keeps
its split-K scratch in a fixed array inside the library instead of taking a
caller-provided workspace.  This test checks, on two calls in a row of one
batch and then a different batch (so later calls run over the earlier
calls' leftover scratch contents), that its output is bit-identical to the
workspace entry point's: both run the same kernel with the same grid and
work split, and the split-K merge order is fixed, so the bits must agree
(tighter than the 2e-3 tolerance of the other decode tests).  The file
sorts last so that a run that stops at the first failure has already run
every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_fn(lib):
    f = lib.vmps_paged_decode_attention_noalloc
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    f.restype = i32
    f.argtypes = [vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, ctypes.c_float, i32, vp]
    return f


def _case(seed, B, n_q, n_kv, D, lo, hi, nb, dev):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(lo, hi + 1, size=B)
    pages = (ctx + 15) // 16
    perm = rng.permutation(nb)
    bt = np.zeros((B, int(pages.max())), np.int32)
    off = 0
    for i, p in enumerate(pages):
        bt[i, :p] = perm[off:off + p]
        off += p
    g = torch.Generator(device=dev).manual_seed(seed)
    pool = torch.randn((nb, 2, 16, n_kv, D), generator=g, device=dev).half()
    q = torch.randn((B, n_q, D), generator=g, device=dev).half()
    return q, pool, torch.from_numpy(bt).to(dev), torch.from_numpy(ctx.astype(np.int32)).to(dev)


def test_noalloc_matches_workspace_entry_point_twice():
    from vllm_mps_b200 import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = K.load_library()
    fn = _noalloc_fn(lib)
    cases = [_case(21, 64, 32, 4, 64, 1, 2048, 16384, dev),   # C1-shaped, many split sequences
             _case(22, 9, 32, 4, 64, 1, 700, 1024, dev)]      # smaller batch over stale scratch
    for q, pool, bt, sl in cases:
        B, n_q, D = q.shape
        n_kv = pool.shape[3]
        ref = K.paged_decode_attention(q, pool, bt, sl)
        for _ in range(2):
            out = torch.full_like(q, float("nan"))
            stream = torch.cuda.current_stream(dev).cuda_stream
            rc = fn(out.data_ptr(), q.data_ptr(), pool.data_ptr(), bt.data_ptr(), bt.shape[1],
                    sl.data_ptr(), B, n_q, n_kv, D, 16, pool.shape[0], 1.0 / np.sqrt(D), 0,
                    stream)
            assert rc == 0, lib.vmps_last_error()
            torch.cuda.synchronize(dev)
            assert K.error_word(dev) == 0
            assert torch.equal(out, ref), (out.float() - ref.float()).abs().max()


def test_noalloc_rejects_calls_beyond_the_scratch_size():
    """16 query heads per kv head need ~10.8 MB of scratch on a 148-SM B200 (> 8 MiB)."""
    from vllm_mps_b200 import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = K.load_library()
    fn = _noalloc_fn(lib)
    need = lib.vmps_paged_decode_workspace_bytes(8, 64, 4, 64, 0)
    assert need > 8 << 20
    q, pool, bt, sl = _case(23, 8, 64, 4, 64, 1, 300, 256, dev)
    out = torch.zeros_like(q)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = fn(out.data_ptr(), q.data_ptr(), pool.data_ptr(), bt.data_ptr(), bt.shape[1],
            sl.data_ptr(), 8, 64, 4, 64, 16, pool.shape[0], 0.125, 0, stream)
    assert rc == -4  # VMPS_ERR_WORKSPACE, rejected on the host
    assert b"scratch" in lib.vmps_last_error()
    torch.cuda.synchronize(dev)
    assert torch.count_nonzero(out) == 0  # nothing was launched
