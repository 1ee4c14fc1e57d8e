"""Sampler kernels: the ``SamplerBackend`` interface, its registry and its backends: ``b200``
(the fused sm_100a kernel) and ``reference`` (vinfer's own PyTorch sampler)."""

from vinfer_b200.kernels.sampler.base import SAMPLER, SamplerBackend
from vinfer_b200.kernels.sampler.b200 import B200Sampler
from vinfer_b200.kernels.sampler.reference import ReferenceSampler

__all__ = ["SAMPLER", "B200Sampler", "ReferenceSampler", "SamplerBackend"]
