"""The sampler backend interface and its registry (a new op family for vinfer's registry).

The interface keeps the reference sampler's call, ``sample(logits, params, seed, position)
-> int`` (``src/vinfer/runtime/sampler.py:68-77``, called per decode step at
``src/vinfer/runtime/generate.py:129``), and adds the batched form the B200 kernel is built
for: one call samples a batch of rows with per-row parameters, per-row token-count histories
and one caller uniform per row, leaving the ids on the device.
"""

from __future__ import annotations

from typing import Protocol

import torch

from vinfer_b200.registry import BackendRegistry
from vinfer_b200.sampling import RowParams, SamplingParams, TokenHistogram


class SamplerBackend(Protocol):
    def sample(self, logits: torch.Tensor, params: SamplingParams, seed: int,
               position: int) -> int:
        """One token id from ``logits`` ``[vocab]`` for the token at ``position``."""
        ...

    def sample_batch(
        self,
        logits: torch.Tensor,
        params: RowParams,
        uniforms: torch.Tensor,
        history: TokenHistogram | None = None,
        out: torch.Tensor | None = None,
        probs_out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Token ids ``int32 [B]`` for ``logits`` ``[B, vocab]`` (row stride may exceed vocab),
        with per-row ``params``, ``uniforms`` ``float32 [B]`` in ``[0, 1)`` and optional
        per-row histories. ``probs_out`` ``float32 [B, vocab]``, if given, receives the final
        probabilities (for parity checks)."""
        ...


SAMPLER: BackendRegistry[SamplerBackend] = BackendRegistry("sampler")
