"""Adapter interface (same as the reference's models/base_adapter.py:18-47)."""

from __future__ import annotations

from abc import ABC, abstractmethod

import torch


class BaseModelAdapter(ABC):
    @abstractmethod
    def load(self, model_config, kv_cache_manager, memory_pool) -> None:
        """Load weights and inject PagedAttentionLayers."""

    @abstractmethod
    def forward_single_token(self, token_id: int, position_id: int, seq_id: int) -> torch.Tensor:
        """Logits ``(vocab,)`` of one token."""

    @abstractmethod
    def get_tokenizer(self):
        """The tokenizer (may be None for random-init models)."""

    @property
    @abstractmethod
    def model_name(self) -> str:
        """Model identifier."""
