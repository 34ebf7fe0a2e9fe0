"""The batched temperature / top-k / top-p sampler on device tensors.

The reference samples one row at a time on its own device
(model/sampler.py:36-59): divide by the temperature, keep every logit >= the
k-th largest, drop sorted tokens whose cumulative probability before them
is >= top_p, sample from the softmax.  Here all sampled rows of a batch go
through one sort on the GPU.  Checked against a CPU restatement of the
reference's per-row steps on float32 logits: the set of surviving tokens is
identical and their probabilities agree to 1e-6; a device generator gives
each row that distribution (frequencies within sampling noise); greedy rows
take the first index of the maximum.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _reference_row(l, p):
    """The reference's per-row filter, on the CPU (model/sampler.py:36-59)."""
    l = l / p.temperature
    if p.top_k > 0:
        th = torch.topk(l, min(p.top_k, l.numel())).values[-1]
        l = torch.where(l < th, torch.tensor(float("-inf")), l)
    if p.top_p < 1.0:
        sl, si = torch.sort(l, descending=True)
        pr = F.softmax(sl, -1)
        sl = sl.masked_fill(torch.cumsum(pr, -1) - pr >= p.top_p, float("-inf"))
        l = torch.zeros_like(l).scatter_(-1, si, sl)
    return l


def _params():
    from vllm_mps_b200.core.sequence import SamplingParams

    return [SamplingParams(temperature=0.7, top_k=5), SamplingParams(temperature=1.3, top_p=0.6),
            SamplingParams(temperature=1.0, top_k=50, top_p=0.8),
            SamplingParams(temperature=0.5, top_k=1), SamplingParams(temperature=2.0),
            SamplingParams(temperature=1.0, top_p=0.95), SamplingParams(temperature=0.9, top_k=32000),
            SamplingParams(temperature=1.1, top_k=7, top_p=0.3)]


def test_filter_masks_match_reference_rows():
    from vllm_mps_b200.model.sampler import Sampler

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(8, 32000, generator=g) * 3.0
    params = _params()
    got = Sampler().filtered_logits(logits.to(dev), params).cpu()
    for r, p in enumerate(params):
        ref = _reference_row(logits[r], p)
        keep_ref, keep = torch.isfinite(ref), torch.isfinite(got[r])
        assert torch.equal(keep, keep_ref), (r, int(keep.sum()), int(keep_ref.sum()))
        torch.testing.assert_close(F.softmax(got[r], -1), F.softmax(ref, -1), atol=1e-6, rtol=0)


def test_device_sampling_distribution_and_greedy_rows():
    from vllm_mps_b200.core.sequence import SamplingParams
    from vllm_mps_b200.model.sampler import Sampler

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(4, 64, generator=g)
    logits[3, 10] = logits[3, 20] = logits[3].max() + 1.0  # tie: first index wins
    params = [SamplingParams(temperature=0.7, top_k=5), SamplingParams(temperature=1.3, top_p=0.6),
              SamplingParams(temperature=1.0, top_k=10, top_p=0.8), SamplingParams(temperature=0.0)]
    want = [F.softmax(_reference_row(logits[r], params[r]), -1) for r in range(3)]
    gen = torch.Generator(device=dev).manual_seed(2)
    n = 4000
    counts = torch.zeros(4, 64)
    batch = logits.to(dev).repeat(n, 1)
    toks = Sampler().sample_rows(batch, params * n, gen)
    for i, t in enumerate(toks):
        counts[i % 4, t] += 1
    for r in range(3):
        emp = counts[r] / n
        assert torch.equal(emp > 0, want[r] > 0), r
        assert (emp - want[r]).abs().max() < 0.03, r
    assert counts[3, 10] == n
