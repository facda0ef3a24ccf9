"""B200-native token sampler for the ecahLang decode loop.

``sample`` / ``Sampler`` / ``torch.ops.ecah.sample`` run the fused sm_100a
kernels of ``lib/libecah_sampler.so`` (C ABI: include/ecah_sampler.h).
"""
from .sampler import PenaltyState, Sampler, launch, new_philox_state, new_workspace  # noqa: F401

__all__ = ["PenaltyState", "Sampler", "launch", "new_philox_state", "new_workspace"]
