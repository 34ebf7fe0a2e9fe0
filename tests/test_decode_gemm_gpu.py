"""The decode GEMM against an fp32 reference of the projections it replaces.

``kernels.decode_gemm(x, w)`` computes ``x @ w.T`` with fp32 accumulation
and one rounding to the 16-bit type: within one 16-bit ulp of the fp32
product (the summation order differs from cuBLAS's), nearly all elements
exactly the rounded fp32 value.  The gated form is compared with
``F.silu(g) * u`` evaluated the way LlamaMLP does it, from the rounded
projections: one ulp of g moves the result by a few ulps at most.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

ULP = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}


def _inputs(dev, dtype, M, N, K, seed, x_pad=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    xb = torch.randn(M, K + x_pad, generator=g, device=dev).to(dtype)
    w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).to(dtype)
    return xb[:, :K], w


def _check_plain(got, x, w):
    ref = x.float() @ w.float().t()
    ulp = ULP[got.dtype]
    torch.testing.assert_close(got.float(), ref, rtol=ulp, atol=ulp)
    same = (got == ref.to(got.dtype)).float().mean().item()
    assert same > 0.99, same


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("N,K", [(2560, 2048), (2048, 2048), (2048, 5632), (24, 64), (136, 576)])
def test_decode_gemm_matches_fp32_reference(cuda_device, dtype, M, N, K):
    from vllm_mps_b200 import kernels as K_

    x, w = _inputs(cuda_device, dtype, M, N, K, seed=M * 131 + N + K)
    got = K_.decode_gemm(x, w)
    torch.cuda.synchronize()
    _check_plain(got, x, w)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,inter,K", [(8, 5632, 2048), (2, 5632, 2048), (5, 64, 1024)])
def test_decode_gemm_gated_epilogue(cuda_device, dtype, M, inter, K):
    from vllm_mps_b200 import kernels as K_

    x, w = _inputs(cuda_device, dtype, M, 2 * inter, K, seed=inter + K + M)
    got = K_.decode_gemm(x, w, silu_mul=True)
    g = (x.float() @ w[:inter].float().t()).to(dtype)
    u = (x.float() @ w[inter:].float().t()).to(dtype)
    want = F.silu(g) * u
    torch.cuda.synchronize()
    ulp = ULP[dtype]
    torch.testing.assert_close(got.float(), want.float(), rtol=4 * ulp, atol=4 * ulp)
    same = (got == want).float().mean().item()
    assert same > 0.97, same


def test_decode_gemm_strided_views_and_chaining(cuda_device):
    """Strided x and out rows; a second call reading the first's output
    (programmatic dependent launch: the second kernel's weight stream starts
    early, its x is read only after the first kernel finishes)."""
    from vllm_mps_b200 import kernels as K_

    dt = torch.float16
    x, w1 = _inputs(cuda_device, dt, 8, 2048, 2048, seed=7, x_pad=64)
    _, w2 = _inputs(cuda_device, dt, 8, 1024, 2048, seed=8)
    big = torch.zeros(8, 2048 + 128, dtype=dt, device=cuda_device)
    y1 = big[:, 64:64 + 2048]
    K_.decode_gemm(x, w1, out=y1)
    y2 = K_.decode_gemm(y1, w2)
    torch.cuda.synchronize()
    _check_plain(y1, x, w1)
    assert big[:, :64].eq(0).all() and big[:, 64 + 2048:].eq(0).all()
    _check_plain(y2, y1, w2)


def test_decode_gemm_rejects_unsupported_shapes(cuda_device):
    from vllm_mps_b200 import kernels as K_

    x = torch.zeros(9, 64, dtype=torch.float16, device=cuda_device)
    w = torch.zeros(8, 64, dtype=torch.float16, device=cuda_device)
    assert not K_.decode_gemm_supported(9, 8, 64)
    with pytest.raises(NotImplementedError):
        K_.decode_gemm(x, w)
    with pytest.raises(NotImplementedError):
        K_.decode_gemm(x[:2, :48], torch.zeros(8, 48, dtype=torch.float16, device=cuda_device))
