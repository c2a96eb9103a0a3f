"""B200-native (sm_100a) SuffixGPU drafter.

Drop-in for the reference ``suffix_gpu`` package's drafter path: the same
``SuffixGPUDrafter`` API, backed by hand-written CUDA kernels reached through
the C ABI in ``include/suffixgpu.h``.
"""

from suffixgpu_b200.proposer import SuffixGPUDrafter

__version__ = "0.1.0"
__all__ = ["SuffixGPUDrafter", "__version__"]
