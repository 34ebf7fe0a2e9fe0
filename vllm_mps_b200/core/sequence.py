"""Requests: sampling settings, one sequence's tokens and state, groups of sequences.

Contract (reference ``core/sequence.py:14-216``): the four statuses, the
``SamplingParams`` fields with their defaults and validity ranges (a bad
value raises ``ValueError``), ``Sequence.add_token`` finishing a sequence
once ``max_tokens`` tokens have been generated, the length getters,
``get_last_token_id`` (``IndexError`` when empty), and ``SequenceGroup``'s
status filters.
"""

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
    """temperature 0 = greedy; top_k 0 = off; top_p 1 = off."""

    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    max_tokens: int = 128
    stop_sequences: list[str] = field(default_factory=list)

    def __post_init__(self) -> None:
        bad = []
        if not self.temperature >= 0.0:
            bad.append(f"temperature={self.temperature} (needs >= 0)")
        if self.top_k < 0:
            bad.append(f"top_k={self.top_k} (needs >= 0)")
        if not 0.0 < self.top_p <= 1.0:
            bad.append(f"top_p={self.top_p} (needs 0 < top_p <= 1)")
        if self.max_tokens < 1:
            bad.append(f"max_tokens={self.max_tokens} (needs >= 1)")
        if bad:
            raise ValueError("invalid sampling parameters: " + ", ".join(bad))


class Sequence:
    """Prompt plus generated token ids of one request, and where it is in its life."""

    def __init__(self, seq_id: int, prompt: str, token_ids: list[int],
                 sampling_params: SamplingParams) -> None:
        self.seq_id = seq_id
        self.prompt = prompt
        self.token_ids = list(token_ids)
        self.prompt_len = len(self.token_ids)
        self.sampling_params = sampling_params
        self.status = SequenceStatus.WAITING
        self.arrival_time = time.time()

    @property
    def output_token_ids(self) -> list[int]:
        """The generated tokens (everything after the prompt)."""
        return self.token_ids[self.prompt_len:]

    def add_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)
        if len(self.token_ids) - self.prompt_len >= self.sampling_params.max_tokens:
            self.status = SequenceStatus.FINISHED

    def get_prompt_len(self) -> int:
        return self.prompt_len

    def get_output_len(self) -> int:
        return len(self.token_ids) - self.prompt_len

    def get_total_len(self) -> int:
        return len(self.token_ids)

    def is_finished(self) -> bool:
        return self.status is SequenceStatus.FINISHED

    def get_last_token_id(self) -> int:
        if not self.token_ids:
            raise IndexError(f"sequence {self.seq_id} has no tokens")
        return self.token_ids[-1]

    def __repr__(self) -> str:
        return (f"<seq {self.seq_id} {self.status.value}: {self.prompt_len} prompt + "
                f"{self.get_output_len()} generated tokens>")


class SequenceGroup:
    """Sequences of one request that share sampling settings."""

    def __init__(self, group_id: int, sequences: list[Sequence],
                 sampling_params: SamplingParams) -> None:
        self.group_id = group_id
        self.sequences = sequences
        self.sampling_params = sampling_params
        self.arrival_time = time.time()

    def get_seqs(self, status: SequenceStatus | None = None) -> list[Sequence]:
        if status is None:
            return list(self.sequences)
        return [s for s in self.sequences if s.status is status]

    def get_num_seqs(self, status: SequenceStatus | None = None) -> int:
        if status is None:
            return len(self.sequences)
        return sum(1 for s in self.sequences if s.status is status)

    def is_finished(self) -> bool:
        return all(s.is_finished() for s in self.sequences)

    def get_max_total_len(self) -> int:
        return max(s.get_total_len() for s in self.sequences)

    def __repr__(self) -> str:
        state = "finished" if self.is_finished() else "live"
        return f"<group {self.group_id}: {len(self.sequences)} sequences, {state}>"
