"""Import-compatible name for the device pool (the reference's module path).

``from vllm_mps.memory.mps_memory_pool import MPSMemoryPool`` keeps working
against this package: the class is the CUDA pool.
"""

from vllm_mps_b200.memory.cuda_memory_pool import CUDAMemoryPool as MPSMemoryPool  # noqa: F401
from vllm_mps_b200.memory.cuda_memory_pool import SwapSpace  # noqa: F401
