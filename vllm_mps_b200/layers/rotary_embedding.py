"""Rotary position embedding (RoPE), HuggingFace-Llama compatible.

Replaces layers/rotary_embedding.py of the reference.  The reference
precomputes fp32 cos/sin tables of shape ``(max_seq_len, d_k)`` and applies
``x*cos + rotate_half(x)*sin`` per sequence in Python (:37-76).  Here the
rotation runs inside kernel 1 (``vmps_rope_reshape_and_cache``) for the
whole batch, evaluating cos/sin of ``position * inv_freq`` on the device for
any position, so no table is needed and positions are not capped by
``max_position_embeddings``.  The ``inv_freq`` vector is built on the host
with the reference's exact fp32 expression (:47-49) so the angles match bit
for bit.
"""

from __future__ import annotations

import torch
import torch.nn as nn


def rope_inv_freq(d_k: int, theta: float) -> torch.Tensor:
    """fp32 ``1 / theta ** (arange(0, d_k, 2) / d_k)`` computed on the CPU.

    Same expression and dtype as the reference (layers/rotary_embedding.py:47-49);
    evaluated with PyTorch's CPU kernels so the table is bit-identical.
    """
    return 1.0 / (theta ** (torch.arange(0, d_k, 2, dtype=torch.float32) / d_k))


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """``cat(-x2, x1)`` over the last dimension (layers/rotary_embedding.py:13-17)."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat([-x2, x1], dim=-1)


class RotaryEmbedding(nn.Module):
    """RoPE parameters of one attention layer.

    Args mirror the reference constructor (layers/rotary_embedding.py:37-43).
    ``max_seq_len`` is kept for API compatibility; the kernels accept any
    non-negative position.
    """

    def __init__(self, d_k: int, max_seq_len: int, theta: float = 10000.0,
                 device: torch.device | None = None) -> None:
        super().__init__()
        self.d_k = d_k
        self.max_seq_len = max_seq_len
        self.theta = theta
        self.register_buffer("inv_freq", rope_inv_freq(d_k, theta).to(device), persistent=False)

    def forward(self, q: torch.Tensor, k: torch.Tensor, position_id: int):
        """Rotate ``q`` (1, n_q, 1, D) and ``k`` (1, n_kv, 1, D) at one position.

        Reference signature (layers/rotary_embedding.py:55-76).  Runs kernel 1
        without a cache write; returns new tensors.
        """
        from vllm_mps_b200.kernels import load_library, _check, dtype_code, _stream

        if not q.is_cuda:
            raise RuntimeError("RotaryEmbedding needs CUDA tensors (no CPU fallback)")
        n_q, n_kv, D = q.shape[1], k.shape[1], q.shape[-1]
        qc = q.reshape(1, n_q * D).contiguous().clone()
        kc = k.reshape(1, n_kv * D).contiguous().clone()
        pos = torch.tensor([position_id], dtype=torch.int32, device=q.device)
        # Rotate k "in place" by treating it as extra query heads.
        both = torch.cat([qc, kc], dim=1)
        lib = load_library()
        dummy = torch.empty(1, 2, 16, n_kv, D, dtype=q.dtype, device=q.device)
        slot = torch.tensor([-1], dtype=torch.int32, device=q.device)
        with torch.cuda.device(q.device):
            rc = lib.vmps_rope_reshape_and_cache(
                both.data_ptr(), both.data_ptr(), both.stride(0), kc.data_ptr(), kc.stride(0),
                kc.data_ptr(), kc.stride(0), pos.data_ptr(), slot.data_ptr(),
                self.inv_freq.data_ptr(), dummy.data_ptr(), 1, n_q + n_kv, n_kv, D, 16, 1,
                dtype_code(q.dtype), _stream(q.device))
        _check(rc, "RotaryEmbedding.forward")
        return (both[:, : n_q * D].reshape(q.shape), both[:, n_q * D:].reshape(k.shape))
