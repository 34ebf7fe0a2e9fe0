"""Configuration constants (same names and defaults as the reference's config.py:10-32).

The reference picks MPS when available; this build's device is CUDA.  The
dimension constants describe the reference's toy model and TinyLlama; the
engine takes its real dimensions from the model configuration.
"""

import torch

# ── Device ────────────────────────────────────────────────────────────────────
DEVICE = "cuda" if torch.cuda.is_available() else "cpu"
DTYPE = torch.float16

# ── Model dimensions (TinyLlama-1.1B) ────────────────────────────────────────
D_MODEL = 2048
N_HEADS = 32
D_K = D_MODEL // N_HEADS
N_LAYERS = 22
VOCAB_SIZE = 32000

# ── Memory pool ───────────────────────────────────────────────────────────────
BLOCK_SIZE = 16             # tokens per physical block
NUM_GPU_BLOCKS = 256        # blocks in the device pool
NUM_CPU_BLOCKS = 128        # blocks in the host (swap) pool
GPU_MEMORY_FRACTION = 0.85  # share of free HBM a sized pool may take

# ── Scheduler ─────────────────────────────────────────────────────────────────
MAX_BATCH_SIZE = 8
MAX_SEQ_LEN = 512
MAX_TOKENS_PER_STEP = 512

# ── Profiler ──────────────────────────────────────────────────────────────────
PROFILER_INTERVAL_SEC = 0.5
