"""Token sampler (same strategies as the reference's model/sampler.py:18-79).

Greedy decoding of a whole batch is one device ``argmax`` (first index on
ties, like ``torch.argmax`` in the reference, :33-34) and one device-to-host
copy of B ids, instead of the reference's per-row ``.item()``
(engine/llm_engine.py:340-344).  Temperature, top-k and top-p follow the
reference's per-row arithmetic, evaluated for all sampled rows at once on the
device.
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
        """One token per row: one argmax for the batch, one batched pass for the rest.

        Rows with ``temperature > 0`` are filtered and sampled together on the
        device (one sort of those rows): the reference's per-row steps
        (model/sampler.py:36-59) -- divide by the temperature; top-k keeps
        every logit >= the k-th largest (ties kept); top-p drops sorted tokens
        whose cumulative probability before them is >= top_p; sample from the
        softmax -- evaluated for all rows at once in sorted order.
        """
        B = logits.size(0)
        if B == 0:
            return []
        out = torch.argmax(logits, dim=-1)
        rows = [i for i, p in enumerate(params) if p.temperature != 0.0]
        if rows:
            dev = logits.device
            idx = torch.tensor(rows, device=dev)
            temp = torch.tensor([params[i].temperature for i in rows], device=dev)
            k = torch.tensor([params[i].top_k for i in rows], device=dev, dtype=torch.long)
            top_p = torch.tensor([params[i].top_p for i in rows], device=dev)
            V = logits.size(-1)
            sv, order = torch.sort(logits[idx].float() / temp[:, None], dim=-1, descending=True)
            kth = sv.gather(1, (k.clamp(1, V) - 1)[:, None])
            kth = torch.where((k > 0)[:, None], kth, torch.full_like(kth, float("-inf")))
            sv = sv.masked_fill(sv < kth, float("-inf"))
            probs = F.softmax(sv, dim=-1)
            cum = torch.cumsum(probs, dim=-1)
            drop = (cum - probs >= top_p[:, None]) & (top_p < 1.0)[:, None]
            sv = sv.masked_fill(drop, float("-inf"))
            pick = torch.multinomial(F.softmax(sv, dim=-1), 1, generator=generator)
            out[idx] = order.gather(1, pick)[:, 0].to(out.dtype)
        return out.tolist()
