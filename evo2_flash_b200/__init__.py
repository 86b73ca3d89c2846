"""evo2_flash_b200: B200-native (sm_100a) Hyena-mixer hot path for Evo 2.

A drop-in for the mixer path of evo2_flash (mixers.py and its Triton kernels):
the same mixer modules, parameter names, paged-state layout and metadata
contract, backed by hand-written CUDA kernels behind a C ABI
(`include/hyena_b200.h`, `_lib/libhyena_b200.so`).
"""

from .forward_context import set_forward_metadata  # noqa: F401
from .mixers import (Bf16Linear, Fp8InProj, HyenaFIRMixer, HyenaIIRMixer,  # noqa: F401
                     HyenaMixerBase)

__all__ = ["HyenaFIRMixer", "HyenaIIRMixer", "HyenaMixerBase", "Fp8InProj", "Bf16Linear",
           "set_forward_metadata"]
