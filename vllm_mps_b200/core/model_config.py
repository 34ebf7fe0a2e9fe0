"""Model configuration (same fields as the reference's core/model_config.py:20-108).

``from_pretrained`` reads a HuggingFace config like the reference (a local
directory works offline).  ``from_hf_config`` builds the same object from an
in-memory ``transformers`` config (random-init models in tests and benches).
On CUDA the dtype is fp16 unless given (the reference: fp16 on MPS, fp32 on
CPU, :71-72).
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch

from vllm_mps_b200.config import BLOCK_SIZE

logger = logging.getLogger(__name__)


@dataclass
class ModelConfig:
    model_name: str
    architecture: str
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_k: int
    n_layers: int
    vocab_size: int
    max_seq_len: int
    rope_theta: float
    dtype: torch.dtype
    device: torch.device

    @classmethod
    def from_hf_config(cls, hf, model_name: str = "model", dtype: torch.dtype | None = None,
                       device: torch.device | str | None = None) -> "ModelConfig":
        """Map a ``transformers`` config to the fields the attention path needs (:50-96)."""
        hidden = getattr(hf, "hidden_size", 2048)
        heads = getattr(hf, "num_attention_heads", 32)
        kv_heads = getattr(hf, "num_key_value_heads", heads) or heads
        arch = "unknown"
        archs = getattr(hf, "architectures", None) or []
        names = [a.lower() for a in archs] + [str(getattr(hf, "model_type", "")).lower()]
        for tag in ("llama", "phi", "mistral"):
            if any(tag in n for n in names):
                arch = tag
                break
        theta = getattr(hf, "rope_theta", None)
        if theta is None:
            rp = getattr(hf, "rope_parameters", None) or {}
            theta = rp.get("rope_theta", 10000.0) if isinstance(rp, dict) else 10000.0
        if device is None:
            device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
        device = torch.device(device)
        if dtype is None:
            dtype = torch.float16 if device.type == "cuda" else torch.float32
        head_dim = getattr(hf, "head_dim", None) or hidden // heads
        return cls(model_name=model_name, architecture=arch, d_model=hidden, n_heads=heads,
                   n_kv_heads=kv_heads, d_k=head_dim,
                   n_layers=getattr(hf, "num_hidden_layers", 22),
                   vocab_size=getattr(hf, "vocab_size", 32000),
                   max_seq_len=getattr(hf, "max_position_embeddings", 2048),
                   rope_theta=float(theta), dtype=dtype, device=device)

    @classmethod
    def from_pretrained(cls, model_name: str) -> "ModelConfig":
        from transformers import AutoConfig

        hf = AutoConfig.from_pretrained(model_name, trust_remote_code=True)
        cfg = cls.from_hf_config(hf, model_name)
        logger.info("ModelConfig: %s arch=%s d_model=%d heads=%d kv_heads=%d d_k=%d layers=%d",
                    model_name, cfg.architecture, cfg.d_model, cfg.n_heads, cfg.n_kv_heads,
                    cfg.d_k, cfg.n_layers)
        return cfg

    def get_kv_cache_config(self) -> dict:
        """Arguments of the KV pool (:100-108)."""
        return {"n_heads": self.n_kv_heads, "d_k": self.d_k, "block_size": BLOCK_SIZE,
                "dtype": self.dtype, "device": self.device}
