"""Request state (same contract as the reference's core/sequence.py:14-216)."""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum


class SequenceStatus(Enum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED = "finished"


@dataclass
class SamplingParams:
    """Sampling configuration (temperature 0 = greedy), validated like :41-61."""

    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    max_tokens: int = 128
    stop_sequences: list[str] = field(default_factory=list)

    def __post_init__(self) -> None:
        if self.temperature < 0.0:
            raise ValueError(f"SamplingParams: temperature must be >= 0.0, got {self.temperature}.")
        if self.top_k < 0:
            raise ValueError(f"SamplingParams: top_k must be >= 0, got {self.top_k}.")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError(f"SamplingParams: top_p must be in (0.0, 1.0], got {self.top_p}.")
        if self.max_tokens < 1:
            raise ValueError(f"SamplingParams: max_tokens must be >= 1, got {self.max_tokens}.")


class Sequence:
    """One request's tokens (prompt + generated) and its lifecycle state."""

    def __init__(self, seq_id: int, prompt: str, token_ids: list[int],
                 sampling_params: SamplingParams) -> None:
        self.seq_id = seq_id
        self.prompt = prompt
        self.token_ids = list(token_ids)
        self.sampling_params = sampling_params
        self.status = SequenceStatus.WAITING
        self.arrival_time = time.time()
        self._prompt_len = len(token_ids)
        self._output_token_ids: list[int] = []

    def add_token(self, token_id: int) -> None:
        """Append a generated token; finish at ``max_tokens`` (:103-113)."""
        self.token_ids.append(token_id)
        self._output_token_ids.append(token_id)
        if len(self._output_token_ids) >= self.sampling_params.max_tokens:
            self.status = SequenceStatus.FINISHED

    def get_prompt_len(self) -> int:
        return self._prompt_len

    def get_output_len(self) -> int:
        return len(self._output_token_ids)

    def get_total_len(self) -> int:
        return len(self.token_ids)

    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    def get_last_token_id(self) -> int:
        if not self.token_ids:
            raise IndexError(f"Sequence [seq={self.seq_id}]: token_ids is empty.")
        return self.token_ids[-1]

    def __repr__(self) -> str:
        return f"Sequence(seq_id={self.seq_id}, status={self.status.value}, total_len={self.get_total_len()})"


class SequenceGroup:
    """Related sequences sharing sampling parameters (:156-216)."""

    def __init__(self, group_id: int, sequences: list[Sequence],
                 sampling_params: SamplingParams) -> None:
        self.group_id = group_id
        self.sequences = sequences
        self.sampling_params = sampling_params
        self.arrival_time = time.time()

    def get_seqs(self, status: SequenceStatus | None = None) -> list[Sequence]:
        if status is None:
            return list(self.sequences)
        return [s for s in self.sequences if s.status == status]

    def get_num_seqs(self, status: SequenceStatus | None = None) -> int:
        return len(self.get_seqs(status))

    def is_finished(self) -> bool:
        return all(s.is_finished() for s in self.sequences)

    def get_max_total_len(self) -> int:
        return max(s.get_total_len() for s in self.sequences)

    def __repr__(self) -> str:
        return (f"SequenceGroup(group_id={self.group_id}, num_seqs={len(self.sequences)}, "
                f"finished={self.is_finished()})")
