"""Kernel 5 (``kernels.batch_gemm``, tcgen05 + cluster split-K) against an fp32 reference.

The kernel accumulates in fp32 and rounds once, like the nn.Linear it
replaces, so every element is within one 16-bit rounding of the fp32 product
(the fp32 summation order differs: a few ulps of fp32, which can move a
rounding by one 16-bit ulp).  Shapes: the Llama-3-8B and TinyLlama
projections at batch 256 (split-K over 2 to 4 CTAs, and unsplit),
batches that are not multiples of 16, strided x and out, a single tile.
Results are bit-identical from run to run (the split partials are summed in
rank order, through the caller's workspace), and the output tiles are
written by TMA stores that clip at M and touch nothing outside ``out``.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [
    # (M, N, K)
    (256, 6144, 4096),   # Llama-3-8B QKV
    (256, 4096, 4096),   # Llama-3-8B O
    (256, 4096, 14336),  # Llama-3-8B down
    (256, 2560, 2048),   # TinyLlama QKV
    (256, 2048, 5632),   # TinyLlama down
    (100, 2048, 2048),   # TinyLlama O, ragged batch
    (17, 11264, 2048),   # TinyLlama [gate; up], 88 tiles
    (1, 128, 64),        # one tile, one K chunk
    (48, 1024, 192),     # three K chunks
]


def _ref(x, w):
    return (x.float() @ w.float().t())


def _check(got, x, w):
    ref = _ref(x, w)
    ulp = 2.0 ** -10 if got.dtype == torch.float16 else 2.0 ** -7
    # One 16-bit rounding of the fp32 result, plus a little for the fp32 order.
    torch.testing.assert_close(got.float(), ref, rtol=1.01 * ulp, atol=1e-4)
    same = (got == ref.to(got.dtype)).float().mean().item()
    assert same > 0.97, same


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_batch_gemm_matches_fp32(cuda_device, dtype, M, N, K):
    from vllm_mps_b200 import kernels as K_

    g = torch.Generator(device=cuda_device).manual_seed(M * 7 + N + K)
    x = (torch.randn(M, K, generator=g, device=cuda_device) * 0.5).to(dtype)
    w = (torch.randn(N, K, generator=g, device=cuda_device) / K ** 0.5).to(dtype)
    assert K_.batch_gemm_split(M, N, K) >= 1
    out = K_.batch_gemm(x, w)
    _check(out, x, w)
    again = K_.batch_gemm(x, w)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))  # deterministic


def test_batch_gemm_splits_the_narrow_shapes(cuda_device):
    from vllm_mps_b200 import kernels as K_

    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    split = K_.batch_gemm_split(256, 4096, 4096)
    assert 2 <= split <= 4 and 32 * split <= sms
    assert K_.batch_gemm_split(256, 28672, 4096) == 1  # 224 tiles: no split
    assert K_.batch_gemm_split(256, 4096, 100) == 0    # K % 64
    assert K_.batch_gemm_split(257, 4096, 4096) == 0   # M > 256
    assert K_.batch_gemm_split(8, 4000, 4096) == 0     # N % 128
    # The split-K partials go through the caller's workspace: needed exactly
    # when K is split.
    assert K_.batch_gemm_workspace_bytes(256, 4096, 4096, torch.bfloat16) > 0
    assert K_.batch_gemm_workspace_bytes(256, 28672, 4096, torch.bfloat16) == 0
    assert K_.batch_gemm_workspace_bytes(256, 4096, 100, torch.bfloat16) == 0  # not built


def test_batch_gemm_workspace_contract(cuda_device):
    """A split shape with a missing or too-small workspace is rejected on the
    host (VMPS_ERR_WORKSPACE, nothing launched); a caller's own workspace,
    reused across calls, gives the same bits as a fresh one."""
    import ctypes

    from vllm_mps_b200 import kernels as K_

    M, N, K = 256, 4096, 4096
    need = K_.batch_gemm_workspace_bytes(M, N, K, torch.bfloat16)
    assert need > 0 and K_.batch_gemm_split(M, N, K) > 1
    g = torch.Generator(device=cuda_device).manual_seed(9)
    x = (torch.randn(M, K, generator=g, device=cuda_device) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=cuda_device) / K ** 0.5).to(torch.bfloat16)
    lib = K_.load_library()
    out = torch.zeros(M, N, device=cuda_device, dtype=torch.bfloat16)
    small = torch.empty(need - 16, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for ws, nbytes in ((None, 0), (small, need - 16)):
        rc = lib.vmps_batch_gemm(out.data_ptr(), N, x.data_ptr(), K, w.data_ptr(), M, N, K,
                                 None if ws is None else ws.data_ptr(), nbytes, 1, stream)
        assert rc == -4, rc
        assert b"workspace" in lib.vmps_last_error()
    torch.cuda.synchronize(cuda_device)
    assert torch.count_nonzero(out) == 0
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    a = K_.batch_gemm(x, w, workspace=ws)
    b = K_.batch_gemm(x, w, workspace=ws)
    c = K_.batch_gemm(x, w)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert torch.equal(a.view(torch.int16), c.view(torch.int16))
    _check(a, x, w)


def test_batch_gemm_strided_operands(cuda_device):
    from vllm_mps_b200 import kernels as K_

    M, N, K = 40, 1024, 512
    g = torch.Generator(device=cuda_device).manual_seed(5)
    xs = torch.randn(M, K + 64, generator=g, device=cuda_device).to(torch.bfloat16)
    x = xs[:, 32:32 + K]  # rows K + 64 apart, 64-byte offset
    w = torch.randn(N, K, generator=g, device=cuda_device).to(torch.bfloat16) / K ** 0.5
    big = torch.full((M, N + 256), 7.0, device=cuda_device, dtype=torch.bfloat16)
    out = K_.batch_gemm(x, w, out=big[:, 128:128 + N])
    _check(out, x, w)
    assert (big[:, :128] == 7.0).all() and (big[:, 128 + N:] == 7.0).all()  # nothing else written
    with pytest.raises(NotImplementedError):
        K_.batch_gemm(x, w[:1000])  # N % 128
    with pytest.raises(ValueError):
        K_.batch_gemm(x, w.t().contiguous().t())  # w not contiguous
