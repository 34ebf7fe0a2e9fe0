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

    @staticmethod
    def _sorted_filtered(logits: torch.Tensor, params: list[SamplingParams]):
        """Temperature, top-k and top-p of every row at once, in sorted order.

        Returns (values, order): each row's scaled logits sorted descending
        with the dropped tokens at -inf, and the vocab index of each column.
        The reference's per-row steps (model/sampler.py:36-59): divide by
        the temperature; top-k keeps every logit >= the k-th largest (ties
        kept); top-p drops sorted tokens whose cumulative probability before
        them is >= top_p.
        """
        dev = logits.device
        temp = torch.tensor([p.temperature for p in params], device=dev)
        k = torch.tensor([p.top_k for p in params], device=dev, dtype=torch.long)
        top_p = torch.tensor([p.top_p for p in params], device=dev)
        V = logits.size(-1)
        sv, order = torch.sort(logits.float() / temp[:, None], dim=-1, descending=True)
        kth = sv.gather(1, (k.clamp(1, V) - 1)[:, None])
        kth = torch.where((k > 0)[:, None], kth, torch.full_like(kth, float("-inf")))
        sv = sv.masked_fill(sv < kth, float("-inf"))
        probs = F.softmax(sv, dim=-1)
        cum = torch.cumsum(probs, dim=-1)
        drop = (cum - probs >= top_p[:, None]) & (top_p < 1.0)[:, None]
        return sv.masked_fill(drop, float("-inf")), order

    def filtered_logits(self, logits: torch.Tensor, params: list[SamplingParams]) -> torch.Tensor:
        """The logits each row samples from (vocab order, dropped tokens at -inf).

        Every row must have ``temperature > 0``.
        """
        if any(p.temperature == 0.0 for p in params):
            raise ValueError("filtered_logits: greedy rows have no sampling distribution")
        sv, order = self._sorted_filtered(logits, params)
        return torch.full_like(sv, float("-inf")).scatter_(1, order, sv)

    def sample_rows(self, logits: torch.Tensor, params: list[SamplingParams],
                    generator: torch.Generator | None = None) -> list[int]:
        """One token per row: one argmax for the batch, one batched pass for the rest.

        Rows with ``temperature > 0`` are filtered (``_sorted_filtered``) and
        sampled together on the device from the softmax of what is left.
        """
        if logits.size(0) == 0:
            return []
        return self.sample_rows_device(logits, params, generator).tolist()

    def sample_rows_device(self, logits: torch.Tensor, params: list[SamplingParams],
                           generator: torch.Generator | None = None,
                           out: torch.Tensor | None = None) -> torch.Tensor:
        """:meth:`sample_rows` without the device-to-host read: int64 ids on the device.

        ``out`` (int64, ``(B,)``, on the logits' device) receives the ids when
        given; a pipelined engine passes the buffer its next step reads them
        from.  Nothing here waits for the GPU when every row is greedy.
        """
        out = torch.argmax(logits, dim=-1, out=out)
        rows = [i for i, p in enumerate(params) if p.temperature != 0.0]
        if rows:
            idx = torch.tensor(rows, device=logits.device)
            sv, order = self._sorted_filtered(logits[idx], [params[i] for i in rows])
            pick = torch.multinomial(F.softmax(sv, dim=-1), 1, generator=generator)
            out[idx] = order.gather(1, pick)[:, 0].to(out.dtype)
        return out
