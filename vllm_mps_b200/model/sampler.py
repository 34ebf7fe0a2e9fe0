"""Token sampler (same strategies as the reference's model/sampler.py:18-79).

Greedy decoding of a whole batch is one device ``argmax`` (first index on
ties, like ``torch.argmax`` in the reference, :33-34) and one device-to-host
copy of B ids, instead of the reference's per-row ``.item()``
(engine/llm_engine.py:340-344).  Temperature, top-k and top-p follow the
reference's per-row arithmetic on the device.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from vllm_mps_b200.core.sequence import SamplingParams


class Sampler:
    def sample(self, logits: torch.Tensor, sampling_params: SamplingParams) -> int:
        """One token from ``logits`` (vocab,)."""
        return self.sample_rows(logits.unsqueeze(0), [sampling_params])[0]

    def sample_batch(self, logits_batch: torch.Tensor, sampling_params: SamplingParams) -> list[int]:
        """One token per row with shared parameters (:62-79)."""
        return self.sample_rows(logits_batch, [sampling_params] * logits_batch.size(0))

    def sample_rows(self, logits: torch.Tensor, params: list[SamplingParams],
                    generator: torch.Generator | None = None) -> list[int]:
        """One token per row; greedy rows share one argmax and one host copy."""
        B = logits.size(0)
        out = torch.argmax(logits, dim=-1)
        for i, p in enumerate(params):
            if p.temperature != 0.0:
                out[i] = self._sample_row(logits[i], p, generator)
        return out.tolist() if B else []

    @staticmethod
    def _sample_row(logits: torch.Tensor, p: SamplingParams, generator) -> torch.Tensor:
        logits = logits.float() / p.temperature
        if p.top_k > 0:
            k = min(p.top_k, logits.size(-1))
            threshold = torch.topk(logits, k).values[-1]
            logits = torch.where(logits < threshold, torch.full_like(logits, float("-inf")), logits)
        if p.top_p < 1.0:
            sorted_logits, idx = torch.sort(logits, descending=True)
            probs = F.softmax(sorted_logits, dim=-1)
            cum = torch.cumsum(probs, dim=-1)
            sorted_logits = sorted_logits.masked_fill(cum - probs >= p.top_p, float("-inf"))
            logits = torch.full_like(logits, float("-inf")).scatter(-1, idx, sorted_logits)
        probs = F.softmax(logits, dim=-1)
        return torch.multinomial(probs, 1, generator=generator)[0]
