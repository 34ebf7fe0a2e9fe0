"""HuggingFace model adapters (layer injection)."""
