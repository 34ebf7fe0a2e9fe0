"""Architecture router (same as the reference's models/auto_adapter.py:22-61)."""

from __future__ import annotations

import logging

from vllm_mps_b200.core.model_config import ModelConfig

logger = logging.getLogger(__name__)


class AutoAdapter:
    @staticmethod
    def from_pretrained(model_name: str, kv_cache_manager, memory_pool):
        config = ModelConfig.from_pretrained(model_name)
        if config.architecture == "llama":
            from vllm_mps_b200.models.llama_adapter import LlamaAdapter

            adapter = LlamaAdapter(model_name)
        elif config.architecture in ("phi", "mistral"):
            raise NotImplementedError(f"{config.architecture} adapter is not implemented")
        else:
            raise ValueError(f"AutoAdapter: unsupported architecture '{config.architecture}'. "
                             "Supported: llama.")
        adapter.load(config, kv_cache_manager, memory_pool)
        return adapter
