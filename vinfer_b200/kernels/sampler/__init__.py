"""Sampler kernels: the ``SamplerBackend`` interface, its registry and the ``b200`` backend."""

from vinfer_b200.kernels.sampler.base import SAMPLER, SamplerBackend
from vinfer_b200.kernels.sampler.b200 import B200Sampler

__all__ = ["SAMPLER", "B200Sampler", "SamplerBackend"]
