"""Host-side KV-cache bookkeeping (integer slot mapping; no tensors)."""
