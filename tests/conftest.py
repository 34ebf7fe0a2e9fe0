"""Shared test configuration: the ``gpu`` marker and fixture helpers."""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def golden_pool_bits(d) -> np.ndarray:
    """Regenerate the seeded pool of an ``attn_*.npz`` fixture (uint16 bits)."""
    from oracle.paged_attention_oracle import f32_to_bits

    shape = (int(d["num_blocks"]), 2, int(d["block_size"]), int(d["n_kv"]), int(d["D"]))
    rng = np.random.default_rng(int(d["pool_seed"]))
    x = rng.standard_normal(size=shape, dtype=np.float32)
    return f32_to_bits(x, str(d["dtype"]))


def prefill_fixture_inputs(d):
    """q/k/v bits and pool of a ``prefill_*.npz`` fixture, regenerated from its seeds."""
    from oracle.paged_attention_oracle import f32_to_bits, prefill_inputs

    dt = str(d["dtype"])
    rows = int(d["q_lens"].sum())
    q, k, v = prefill_inputs(int(d["input_seed"]), rows, int(d["n_q"]), int(d["n_kv"]),
                             int(d["D"]))
    return f32_to_bits(q, dt), f32_to_bits(k, dt), f32_to_bits(v, dt), golden_pool_bits(d)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def device_error_word_stays_clear(request):
    """After every GPU test the kernels' device error word must be clear.

    Tests that provoke an error on purpose read (and so clear) the word
    themselves; any other bit left set means a kernel skipped an access.
    """
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from vllm_mps_b200 import kernels as K

    word = K.error_word(torch.device("cuda", 0))
    assert word == 0, f"device error word {word} left set by {request.node.name}"
