"""vinfer_b200: a B200-native (sm_100a) token sampler for vinfer.

One fused, memory-bound CUDA pass per batch of logits rows (penalties, temperature, top-k,
softmax, top-p, min-p, inverse-CDF draw), reached through a C ABI
(``include/vinfer_sampler.h``) and registered as the ``b200`` backend of a ``sampler`` op
family with the same registry contract as vinfer's kernel registry.
"""

from vinfer_b200.kernels.sampler import SAMPLER, B200Sampler, SamplerBackend
from vinfer_b200.registry import BackendContext, BackendRegistry
from vinfer_b200.sampling import (
    RowParams,
    SamplingParams,
    SlotHistogram,
    TokenHistogram,
    position_seed,
    position_uniform,
)

__all__ = [
    "SAMPLER",
    "B200Sampler",
    "BackendContext",
    "BackendRegistry",
    "RowParams",
    "SamplerBackend",
    "SamplingParams",
    "SlotHistogram",
    "TokenHistogram",
    "position_seed",
    "position_uniform",
]
