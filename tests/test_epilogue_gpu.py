"""The fused decoder-layer element-wise kernels against the modules they replace.

``kernels.add_rmsnorm`` against ``residual + delta`` followed by transformers'
``LlamaRMSNorm``; ``kernels.silu_mul`` against ``F.silu(gate) * up``.  The
kernels keep the modules' rounding points, so outputs are bit-identical up
to the fp32 summation order of the variance (and CUDA's exp for SiLU): within
two 16-bit ulps, nearly all elements identical.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _close(got: torch.Tensor, want: torch.Tensor) -> None:
    """Within two 16-bit ulps (one rounding of the normalised value can move the
    product with the weight by two), and nearly all elements bit-identical."""
    ulp = 2.0 ** -10 if got.dtype == torch.float16 else 2.0 ** -7
    torch.testing.assert_close(got.float(), want.float(), rtol=2 * ulp, atol=1e-6)
    same = (got.view(torch.int16) == want.view(torch.int16)).float().mean().item()
    assert same > 0.98, same


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,hidden", [(1, 2048), (8, 2048), (256, 4096), (3, 8192)])
def test_add_rmsnorm_matches_llama_rmsnorm(cuda_device, dtype, rows, hidden):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    from vllm_mps_b200 import kernels as K

    g = torch.Generator(device=cuda_device).manual_seed(rows * 7 + hidden)
    res = torch.randn(rows, hidden, generator=g, device=cuda_device).to(dtype)
    delta = torch.randn(rows, hidden, generator=g, device=cuda_device).to(dtype)
    norm = LlamaRMSNorm(hidden, eps=1e-5).to(device=cuda_device, dtype=dtype)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(hidden, generator=g, device=cuda_device) + 0.5)
        want_res = res + delta
        want = norm(want_res)
    got_res = res.clone()
    got = K.add_rmsnorm(got_res, norm.weight.detach(), norm.variance_epsilon, delta=delta)
    torch.cuda.synchronize()
    assert torch.equal(got_res, want_res)  # the residual addition is exact
    _close(got, want)
    # Without delta: the norm alone, residual untouched.
    keep = res.clone()
    got2 = K.add_rmsnorm(keep, norm.weight.detach(), norm.variance_epsilon)
    with torch.no_grad():
        want2 = norm(res)
    assert torch.equal(keep, res)
    _close(got2, want2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,inter", [(1, 5632), (8, 5632), (256, 14336)])
def test_silu_mul_matches_silu_times_up(cuda_device, dtype, rows, inter):
    from vllm_mps_b200 import kernels as K

    g = torch.Generator(device=cuda_device).manual_seed(rows + inter)
    gu = (torch.randn(rows, 2 * inter, generator=g, device=cuda_device) * 3).to(dtype)
    want = F.silu(gu[:, :inter]) * gu[:, inter:]
    got = K.silu_mul(gu)
    torch.cuda.synchronize()
    _close(got, want)


def test_epilogue_argument_checks(cuda_device):
    from vllm_mps_b200 import kernels as K

    x = torch.zeros(4, 12, dtype=torch.float16, device=cuda_device)  # hidden % 8 != 0
    w = torch.ones(12, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError):
        K.add_rmsnorm(x, w, 1e-5)
