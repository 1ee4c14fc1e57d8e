"""The reference sampler's own CPU path, restated in PyTorch for the CPU baseline.

TEST INFRASTRUCTURE ONLY (see ``oracle/sampler_oracle.py``). vinfer's sampler is pure PyTorch
(``src/vinfer/runtime/sampler.py``) and cannot be shipped to the GPU box, so ``bench.py``
times this restatement in its place: the same torch operations in the same order (topk,
masked_fill, softmax, sort, cumsum, scatter, exponential noise from a generator seeded by
``position_seed``, argmax), per row, as ``runtime/generate.py:129`` calls it. It is pinned
bit-exactly to the reference by ``tests/golden/sampler_golden.npz`` (token ids of the
reference's ``sample`` for fixed seeds and positions).

Rows that use features the reference lacks (penalties, min-p) get them applied around the
reference steps with the oracle's definitions, so a penalty workload can be timed too.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle.sampler_oracle import RowParams, position_seed


def reference_filtered_probs(logits: torch.Tensor, temperature: float, top_k: int,
                             top_p: float) -> torch.Tensor:
    """Temperature, top-k and top-p probabilities, float32 (reference ``sampler.py:50-65``)."""
    scaled = logits.float() / temperature
    vocab = scaled.shape[-1]
    if top_k and top_k < vocab:
        kth = torch.topk(scaled, top_k, dim=-1).values[..., -1:]
        scaled = scaled.masked_fill(scaled < kth, float("-inf"))
    probs = torch.softmax(scaled, dim=-1)
    if top_p < 1:
        desc, order = torch.sort(probs, dim=-1, descending=True)
        mass_before = desc.cumsum(-1) - desc
        desc = desc.masked_fill(mass_before >= top_p, 0.0)
        probs = torch.zeros_like(probs).scatter(-1, order, desc)
        probs = probs / probs.sum(-1, keepdim=True)
    return probs


def _race(probs: torch.Tensor, seed: int, position: int) -> int:
    """Exponential-race draw ``argmax(p / E)`` (reference ``sampler.py:73-77``)."""
    gen = torch.Generator(device=probs.device).manual_seed(position_seed(seed, position))
    noise = torch.empty_like(probs).exponential_(generator=gen)
    noise.clamp_min_(torch.finfo(noise.dtype).tiny)
    return int(torch.argmax(probs / noise))


def reference_sample(logits: torch.Tensor, params: RowParams, seed: int, position: int) -> int:
    """One token id, as reference ``sample(logits, params, seed, position)`` returns it."""
    if params.temperature == 0:
        return int(torch.argmax(logits))
    probs = reference_filtered_probs(logits, params.temperature, params.top_k, params.top_p)
    return _race(probs, seed, position)


def extended_sample(logits: torch.Tensor, params: RowParams, seed: int, position: int,
                    hist_ids: np.ndarray | None = None,
                    hist_counts: np.ndarray | None = None) -> int:
    """``reference_sample`` with the build's extensions around it: penalties before the
    reference steps, min-p after them (oracle definitions), same exponential race."""
    x = logits.float()
    if hist_ids is not None and len(hist_ids):
        ids = torch.as_tensor(np.asarray(hist_ids, dtype=np.int64))
        c = torch.as_tensor(np.asarray(hist_counts, dtype=np.float32))
        t = x[ids]
        rep = torch.tensor(params.repetition_penalty, dtype=torch.float32)
        t = torch.where(t > 0, t / rep, t * rep)
        t = t - torch.tensor(params.frequency_penalty, dtype=torch.float32) * c
        t = t - torch.tensor(params.presence_penalty, dtype=torch.float32)
        x = x.clone()
        x[ids] = t
    if params.temperature == 0:
        return int(torch.argmax(x))
    probs = reference_filtered_probs(x, params.temperature, params.top_k, params.top_p)
    if params.min_p > 0:
        probs = probs.masked_fill(probs < params.min_p * probs.max(), 0.0)
        probs = probs / probs.sum()
    return _race(probs, seed, position)
